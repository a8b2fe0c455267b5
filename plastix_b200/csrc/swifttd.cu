// SwiftTD step on the device: TD(lambda) with per-feature meta-learned step
// sizes, one linear value unit fed by N features, every per-feature value a
// connection field in SoA (examples/swifttd/swifttd.cpp:29-209 in the
// reference; its Network::DoStep is plastix.hpp:439-455).
//
// The reference runs three dense sweeps over all N connections per step
// (forward, UpdateIncoming = phase 1, UpdateOutgoing = phase 2) and mutates
// the globals V, Tau, B and VDelta from inside the per-connection policies.
// Only active features (F != 0) contribute to those four sums, so the step is
// restructured around them, three launches per step, each a programmatic
// dependent of the one before (griddepcontrol.wait orders the memory):
//
//   k_td_value   one thread per active feature: V = sum W*F (fp64 partial per
//                CTA in a fixed tree order, CTA partials summed in CTA order
//                by the last CTA to finish), then Loss (Delta, VDeltaPrev).
//                Also the per-tile start offsets into the active list that
//                k_td_dense reads.
//   k_td_terms   one thread per active feature: gathers the four fields phase
//                1 needs for the sums (Z, ZDelta, P, Beta) while k_td_value
//                is still running, then phase 1 for its feature and the
//                Tau = sum exp(Beta')*F*F, B = sum Z'*F and VDelta =
//                sum DeltaW*F reductions, same scheme as V.
//   k_td_dense   one pass over all N features: phase 1 and phase 2 fused,
//                8 fields read through a bulk-copy ring and 10 written with
//                128-bit stores; its first copies overlap k_td_terms.
//                ResetGlobal (VOld = V) at the end.
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

constexpr int kTdThreads = 256;          // dense pass CTA
constexpr int kTdTile = 1024;            // features per dense tile (float4/thread)
constexpr int kTdAThreads = 256;         // active-set CTAs: one thread per feature
constexpr uint32_t kTdAMaxBlocks = 2048; // beyond 524,288 active features, threads loop

struct TdGlobals {
  float gamma, lambda, eta, eta_min, decay, meta;
  float v, v_old, delta, v_delta_prev, v_delta, tau, b;
};
static_assert(sizeof(TdGlobals) == sizeof(plx_td_globals), "globals layout");

struct TdScratch {
  uint32_t* tickets;  // [0] dense tile queue, [1] dense CTAs done, [2] value CTAs
                      // done, [3] terms CTAs done; all zero between steps
  double* part;       // [kTdAMaxBlocks][4]: V, Tau, B, VDelta partial per CTA
  uint32_t* start;    // [n_tiles + 1]
};

struct TdFields {
  float* f[PLX_TD_NUM_FIELDS];
};

enum : int { W = 0, Z, ZD, DW, H, HOLD, HTEMP, ZBAR, P, BETA };

inline uint64_t td_scratch_layout(uint64_t n_features, uint64_t* off_part,
                                  uint64_t* off_start) {
  const uint64_t tiles = (n_features + kTdTile - 1) / kTdTile;
  *off_part = 256;  // after the tickets
  *off_start = *off_part + 32ull * kTdAMaxBlocks;
  return (*off_start + 4 * (tiles + 1) + 255) & ~uint64_t(255);
}

__host__ __device__ inline uint32_t td_active_blocks(uint64_t n_active) {
  const uint64_t b = (n_active + kTdAThreads) / kTdAThreads;  // covers k = n_active
  return (uint32_t)(b < kTdAMaxBlocks ? b : kTdAMaxBlocks);
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
template <int NV, int NT>
__device__ __forceinline__ void block_sum(double (&v)[NV], double (*s_red)[NT / 32]) {
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
      for (int k = 0; k < NT / 32; ++k) s += s_red[j][k];
      v[j] = s;
    }
  }
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// Tile start offsets for position k of the active list (k == a.k is the
// sentinel): start[t] = first position whose feature lies in tile >= t.
// Returns false for an unsorted or out-of-range entry.
__device__ __forceinline__ bool td_tile_starts(const TdActiveArgs& a, uint64_t k) {
  uint64_t t_lo, t_hi;
  const uint32_t prev = k ? a.idx[k - 1] : 0;
  if (k < a.k) {
    const uint32_t cur = a.idx[k];
    if (cur >= a.n || (k && prev >= cur)) return false;
    t_lo = k ? (uint64_t)prev / kTdTile + 1 : 0;
    t_hi = (uint64_t)cur / kTdTile;
  } else {
    const uint64_t pv = prev < a.n ? prev : a.n - 1;  // n >= 1
    t_lo = k ? pv / kTdTile + 1 : 0;
    t_hi = a.n_tiles;
  }
  for (uint64_t t = t_lo; t <= t_hi && t <= a.n_tiles; ++t) a.s.start[t] = (uint32_t)k;
  return true;
}

// True in every thread of the last CTA of the grid to get here; that CTA
// then sees the partials the others stored before arriving.
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

__global__ void __launch_bounds__(kTdAThreads) k_td_value(TdActiveArgs a, TdFields fl) {
  __shared__ double s_red[1][kTdAThreads / 32];
  // The previous step's dense pass must be complete (and visible) before W is
  // read; only then may k_td_terms start gathering.
  grid_dependency_wait();
  grid_dependents_launch();
  const uint64_t nthr = (uint64_t)gridDim.x * kTdAThreads;
  const uint64_t gtid = (uint64_t)blockIdx.x * kTdAThreads + threadIdx.x;
  bool bad = false;
  double v[1] = {0.0};
  for (uint64_t k = gtid; k <= a.k; k += nthr) {
    bad |= !td_tile_starts(a, k);
    if (k < a.k) {
      const uint32_t i = a.idx[k];
      if (i < a.n) v[0] += (double)__fmul_rn(fl.f[W][i], active_value(a, (uint32_t)k));
    }
  }
  if (bad) record_status(a.status, kStatusBadIndex);
  block_sum<1, kTdAThreads>(v, s_red);
  if (threadIdx.x == 0) a.s.part[(uint64_t)blockIdx.x * 4] = v[0];
  if (!last_block(&a.s.tickets[2])) return;
  __syncthreads();  // s_red is reused
  // CTA partials summed by a fixed tree: thread j takes CTAs j, j + 256, ...
  v[0] = 0.0;
  for (uint32_t b = threadIdx.x; b < gridDim.x; b += kTdAThreads)
    v[0] += __ldcg(&a.s.part[(uint64_t)b * 4]);
  block_sum<1, kTdAThreads>(v, s_red);
  if (threadIdx.x == 0) {
    // DoForwardPass Apply (swifttd.cpp:81-84) and Loss (:90-100).
    TdGlobals& g = *a.g;
    g.v = (float)v[0];
    g.delta = __fsub_rn(__fadd_rn(*a.reward, __fmul_rn(g.gamma, g.v)), g.v_old);
    g.v_delta_prev = g.v_delta;
    g.v_delta = 0.0f;
    g.tau = 0.0f;
    g.b = 0.0f;
    if (a.v_out) *a.v_out = g.v;
    a.s.tickets[2] = 0;
  }
}

__global__ void __launch_bounds__(kTdAThreads) k_td_terms(TdActiveArgs a, TdFields fl) {
  __shared__ double s_red[3][kTdAThreads / 32];
  const uint64_t nthr = (uint64_t)gridDim.x * kTdAThreads;
  const uint64_t gtid = (uint64_t)blockIdx.x * kTdAThreads + threadIdx.x;
  // Gather this thread's first feature before waiting for k_td_value: the
  // fields are not written by it, and the step before is complete (k_td_value
  // let this kernel start only after its own wait). Phase 1 needs Z, ZDelta,
  // P and Beta for the sums (W, H, HTemp, ZBar do not enter them).
  const bool first = gtid < a.k;
  const uint32_t i0 = first ? a.idx[gtid] : 0xFFFFFFFFu;
  const bool ok0 = i0 < a.n;
  float z0 = ok0 ? fl.f[Z][i0] : 0.0f, zd0 = ok0 ? fl.f[ZD][i0] : 0.0f;
  float p0 = ok0 ? fl.f[P][i0] : 0.0f, be0 = ok0 ? fl.f[BETA][i0] : 0.0f;
  const float f0 = first ? active_value(a, (uint32_t)gtid) : 0.0f;
  grid_dependency_wait();  // Delta and VDeltaPrev of this step
  grid_dependents_launch();
  const TdConst c = td_const(*a.g);
  double t[3] = {0.0, 0.0, 0.0};
  auto term = [&](float f, float z, float zd, float p, float beta) {
    float w = 0.0f, dw, h = 0.0f, h_old, h_temp = 0.0f, z_bar = 0.0f;
    const float eb = td_phase1(c, w, z, zd, dw, h, h_old, h_temp, z_bar, p, beta);
    t[0] += (double)__fmul_rn(__fmul_rn(eb, f), f);  // Tau, swifttd.cpp:148
    t[1] += (double)__fmul_rn(z, f);                 // B, :149
    t[2] += (double)__fmul_rn(dw, f);                // VDelta, :167
  };
  if (ok0) term(f0, z0, zd0, p0, be0);
  for (uint64_t k = gtid + nthr; k < a.k; k += nthr) {
    const uint32_t i = a.idx[k];
    if (i < a.n)
      term(active_value(a, (uint32_t)k), fl.f[Z][i], fl.f[ZD][i], fl.f[P][i], fl.f[BETA][i]);
  }
  block_sum<3, kTdAThreads>(t, s_red);
  if (threadIdx.x == 0)
    for (int j = 0; j < 3; ++j) a.s.part[(uint64_t)blockIdx.x * 4 + 1 + j] = t[j];
  if (!last_block(&a.s.tickets[3])) return;
  t[0] = t[1] = t[2] = 0.0;
  for (uint32_t b = threadIdx.x; b < gridDim.x; b += kTdAThreads)
    for (int j = 0; j < 3; ++j) t[j] += __ldcg(&a.s.part[(uint64_t)b * 4 + 1 + j]);
  __syncthreads();  // s_red is reused
  block_sum<3, kTdAThreads>(t, s_red);
  if (threadIdx.x == 0) {
    a.g->tau = (float)t[0];
    a.g->b = (float)t[1];
    a.g->v_delta = (float)t[2];
    a.s.tickets[3] = 0;
  }
}

__device__ __forceinline__ void st4(float* p, float4 v) {
  __stcs(reinterpret_cast<float4*>(p), v);
}

// Dense pass layout. Tiles of kTdTile features are handed out by an atomic
// queue (so the ~4096 tiles of a 4M-feature step spread evenly over the
// resident CTAs). Per tile, thread 0 issues eight 4 KB bulk copies (the fields
// the update reads) into a kTdStages-deep shared ring, kTdStages - 1 tiles
// ahead of the compute; each thread then updates four features from shared
// memory and writes the ten fields with 128-bit stores. F comes from a shared
// slot table filled one tile ahead from the sorted active list: slot o holds
// the position k in the active list of feature tile*kTdTile + o. A CTA takes
// tiles in increasing order, so entries left from its earlier tiles hold
// positions below this tile's range [ka, kb) and read as inactive: no
// clearing between tiles. The partial last tile (n % kTdTile features) takes
// a scalar path with no bulk copies.
constexpr int kTdStages = 3;
constexpr int kTdLoadFields = 8;
constexpr uint32_t kTdNoTile = 0xFFFFFFFFu;

struct TdDenseSmem {
  float in[kTdStages][kTdLoadFields][kTdTile];
  uint32_t slot[2][kTdTile];
  uint32_t range[2][2];  // [ka, kb) of the tile in each slot buffer
  uint32_t tile_of[kTdStages];
  uint64_t full[kTdStages];
};

// The fields the update reads, in ring order: W, Z, ZD, H, HTEMP, ZBAR, P, BETA
// (DeltaW and HOld are written only).
__host__ __device__ constexpr int td_load_field(int f) {
  return f < 3 ? f : (f == 3 ? int(H) : f + 2);
}
static_assert(td_load_field(4) == HTEMP && td_load_field(7) == BETA, "ring order");

#define PLX_TD_LANE(comp)                                                          \
  do {                                                                             \
    float dw_, h_old_;                                                             \
    td_phase1(c, vw.comp, vz.comp, vzd.comp, dw_, vh.comp, h_old_, vht.comp,       \
              vzb.comp, vp.comp, vbe.comp);                                        \
    td_phase2(c, fv.comp, vz.comp, vzd.comp, vh.comp, h_old_, vht.comp, vzb.comp,  \
              vp.comp, vbe.comp);                                                  \
    vdw.comp = dw_;                                                                \
    vho.comp = h_old_;                                                             \
  } while (0)

__global__ void __launch_bounds__(kTdThreads, 2)
    k_td_dense(TdActiveArgs a, TdFields fl, uint64_t timeout_ns) {
  extern __shared__ __align__(128) unsigned char td_smem_raw[];
  TdDenseSmem& sm = *reinterpret_cast<TdDenseSmem*>(td_smem_raw);
  const uint32_t tid = threadIdx.x;
  const uint64_t n_full = a.n / kTdTile;  // tiles fed by bulk copies
  uint32_t* queue = &a.s.tickets[0];

  for (uint32_t o = tid; o < 2 * kTdTile; o += kTdThreads) (&sm.slot[0][0])[o] = kTdNoTile;
  if (tid == 0) {
    for (int st = 0; st < kTdStages; ++st) mbar_init(&sm.full[st], 1);
    mbar_init_fence();
  }
  __syncthreads();

  // Thread 0: take the next tile from the queue and start its copies.
  auto issue = [&](uint32_t j) {
    const uint32_t st = j % kTdStages;
    const uint32_t t = atomicAdd(queue, 1u);
    sm.tile_of[st] = t < a.n_tiles ? t : kTdNoTile;
    if (t < n_full) {
      mbar_arrive_expect_tx(&sm.full[st], kTdLoadFields * kTdTile * 4);
      const uint64_t base = (uint64_t)t * kTdTile;
#pragma unroll
      for (int f = 0; f < kTdLoadFields; ++f)
        bulk_load(sm.in[st][f], fl.f[td_load_field(f)] + base, kTdTile * 4, &sm.full[st]);
    } else {
      mbar_arrive_expect_tx(&sm.full[st], 0);  // completes the phase at once
    }
  };
  // All threads: the active features of tile t into slot buffer `buf`.
  auto scatter = [&](uint32_t t, uint32_t buf) {
    if (t == kTdNoTile) return;
    const uint64_t base = (uint64_t)t * kTdTile;
    const uint32_t ka = min(a.s.start[t], a.k);
    const uint32_t kb = max(min(a.s.start[t + 1], a.k), ka);
    if (tid == 0) {
      sm.range[buf][0] = ka;
      sm.range[buf][1] = kb;
    }
    for (uint32_t k = ka + tid; k < kb; k += kTdThreads) {
      const uint64_t off = (uint64_t)a.idx[k] - base;
      if (off < kTdTile) sm.slot[buf][off] = k;
    }
  };
  // F of the feature in slot o of buffer buf.
  auto feature = [&](uint32_t buf, uint32_t o) {
    const uint32_t k = sm.slot[buf][o];
    return (k >= sm.range[buf][0] && k < sm.range[buf][1]) ? active_value(a, k) : 0.0f;
  };

  // Copies of the first tiles may start before k_td_terms has finished:
  // the kernels before only read the fields. The queue was reset by the
  // previous dense pass, which completed before k_td_value let the next
  // kernels start.
  if (tid == 0)
    for (uint32_t j = 0; j + 1 < kTdStages; ++j) issue(j);
  grid_dependency_wait();  // start offsets and globals of this step
  const TdConst c = td_const(*a.g);
  __syncthreads();
  scatter(sm.tile_of[0], 0);
  __syncthreads();

  uint32_t j = 0;
  bool failed = false;
  for (;; ++j) {
    const uint32_t st = j % kTdStages;
    const uint32_t t = sm.tile_of[st];
    if (t == kTdNoTile) break;  // uniform: every thread read the same slot
    if (tid == 0) issue(j + kTdStages - 1);
    scatter(sm.tile_of[(j + 1) % kTdStages], (j + 1) & 1);
    const bool ok = mbar_wait_bounded(&sm.full[st], (j / kTdStages) & 1, timeout_ns);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    const uint32_t buf = j & 1;
    const uint64_t base = (uint64_t)t * kTdTile;
    const uint32_t o = 4 * tid;
    if (t < n_full) {
      float4 vw = *reinterpret_cast<const float4*>(&sm.in[st][0][o]);
      float4 vz = *reinterpret_cast<const float4*>(&sm.in[st][1][o]);
      float4 vzd = *reinterpret_cast<const float4*>(&sm.in[st][2][o]);
      float4 vh = *reinterpret_cast<const float4*>(&sm.in[st][3][o]);
      float4 vht = *reinterpret_cast<const float4*>(&sm.in[st][4][o]);
      float4 vzb = *reinterpret_cast<const float4*>(&sm.in[st][5][o]);
      float4 vp = *reinterpret_cast<const float4*>(&sm.in[st][6][o]);
      float4 vbe = *reinterpret_cast<const float4*>(&sm.in[st][7][o]);
      const float4 fv = make_float4(feature(buf, o), feature(buf, o + 1),
                                    feature(buf, o + 2), feature(buf, o + 3));
      float4 vdw, vho;
      PLX_TD_LANE(x);
      PLX_TD_LANE(y);
      PLX_TD_LANE(z);
      PLX_TD_LANE(w);
      const uint64_t i0 = base + o;
      st4(fl.f[W] + i0, vw);
      st4(fl.f[Z] + i0, vz);
      st4(fl.f[ZD] + i0, vzd);
      st4(fl.f[DW] + i0, vdw);
      st4(fl.f[H] + i0, vh);
      st4(fl.f[HOLD] + i0, vho);
      st4(fl.f[HTEMP] + i0, vht);
      st4(fl.f[ZBAR] + i0, vzb);
      st4(fl.f[P] + i0, vp);
      st4(fl.f[BETA] + i0, vbe);
    } else {
      // Partial last tile: plain loads and stores, feature by feature.
      for (uint32_t q = 0; q < 4; ++q) {
        const uint64_t i = base + o + q;
        if (i >= a.n) break;
        float* const* f = fl.f;
        const float fq = feature(buf, o + q);
        float w1 = f[W][i], z1 = f[Z][i], zd1 = f[ZD][i], dw1, h1 = f[H][i], ho1,
              ht1 = f[HTEMP][i], zb1 = f[ZBAR][i], p1 = f[P][i], be1 = f[BETA][i];
        td_phase1(c, w1, z1, zd1, dw1, h1, ho1, ht1, zb1, p1, be1);
        td_phase2(c, fq, z1, zd1, h1, ho1, ht1, zb1, p1, be1);
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
    __syncthreads();  // stage st and slot buffer `buf` are free again
  }
  if (failed && tid == 0) {
    // Let this CTA's copies still in flight land before shared memory is
    // released: the stages of slots j .. j + kTdStages - 1 may be pending
    // (slot j + kTdStages - 1 was issued at the top of this iteration).
    record_status(a.status, kStatusTimeout);
    for (uint32_t q = j; q < j + kTdStages; ++q)
      if (!mbar_wait_bounded(&sm.full[q % kTdStages], (q / kTdStages) & 1, timeout_ns)) break;
  }
  // After a normal exit the slots past the last one hold no copies: their
  // queue tickets were past the last tile and their phases completed on
  // arrival. The last CTA to finish resets the queue for the next step.
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&a.s.tickets[1], 1u) == gridDim.x - 1) {
      a.s.tickets[0] = 0;
      a.s.tickets[1] = 0;
    }
  }
  // ResetGlobal (swifttd.cpp:189-191). No block of this kernel reads V or VOld.
  if (!failed && blockIdx.x == 0 && tid == 0) a.g->v_old = a.g->v;
}
#undef PLX_TD_LANE

}  // namespace
}  // namespace plx

using namespace plx;

extern "C" uint64_t plx_swifttd_scratch_bytes(uint64_t n_features, uint32_t max_active) {
  (void)max_active;  // the partials area is sized for the largest grid
  uint64_t op, os;
  return td_scratch_layout(n_features, &op, &os);
}

namespace {

constexpr int kTdRunReduce = 1;  // k_td_value + k_td_terms
constexpr int kTdRunApply = 2;   // k_td_dense

int td_launch(plx_ctx* ctx, uint64_t n_features, float* const* fields,
              const uint32_t* active_idx, const float* active_val, uint32_t n_active,
              const float* reward, plx_td_globals* globals, float* v_out, void* scratch,
              uint64_t scratch_bytes, int parts) {
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
  uint64_t op, os;
  const uint64_t need = td_scratch_layout(n_features, &op, &os);
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
  a.s.part = reinterpret_cast<double*>(s + op);
  a.s.start = reinterpret_cast<uint32_t*>(s + os);
  a.n_tiles = (n_features + kTdTile - 1) / kTdTile;
  a.status = ctx->d_status;

  static thread_local int smem_set_device = -1;
  const size_t smem = sizeof(TdDenseSmem);
  if (smem_set_device != ctx->device) {
    PLX_TRY_CUDA(cudaFuncSetAttribute(k_td_dense, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    smem_set_device = ctx->device;
  }

  // Every launch is a programmatic dependent of the kernel before it in the
  // stream (griddepcontrol.wait in each orders the memory).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = ctx->stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (parts & kTdRunReduce) {
    cfg.gridDim = dim3(td_active_blocks(n_active));
    cfg.blockDim = dim3(kTdAThreads);
    cfg.dynamicSmemBytes = 0;
    PLX_TRY_CUDA(cudaLaunchKernelEx(&cfg, k_td_value, a, fl));
    PLX_TRY_CUDA(cudaLaunchKernelEx(&cfg, k_td_terms, a, fl));
  }
  if (parts & kTdRunApply) {
    cfg.gridDim =
        dim3((unsigned)std::min<uint64_t>(a.n_tiles, 2ull * (uint64_t)ctx->num_sms));
    cfg.blockDim = dim3(kTdThreads);
    cfg.dynamicSmemBytes = smem;
    PLX_TRY_CUDA(cudaLaunchKernelEx(&cfg, k_td_dense, a, fl, (uint64_t)ctx->timeout_ns));
  }
  return PLX_OK;
}

}  // namespace

extern "C" int plx_swifttd_step(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                                const uint32_t* active_idx, const float* active_val,
                                uint32_t n_active, const float* reward,
                                plx_td_globals* globals, float* v_out, void* scratch,
                                uint64_t scratch_bytes) {
  return td_launch(ctx, n_features, fields, active_idx, active_val, n_active, reward, globals,
                   v_out, scratch, scratch_bytes, kTdRunReduce | kTdRunApply);
}

extern "C" int plx_swifttd_reduce(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                                  const uint32_t* active_idx, const float* active_val,
                                  uint32_t n_active, const float* reward,
                                  plx_td_globals* globals, float* v_out, void* scratch,
                                  uint64_t scratch_bytes) {
  return td_launch(ctx, n_features, fields, active_idx, active_val, n_active, reward, globals,
                   v_out, scratch, scratch_bytes, kTdRunReduce);
}

extern "C" int plx_swifttd_apply(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                                 const uint32_t* active_idx, const float* active_val,
                                 uint32_t n_active, plx_td_globals* globals, void* scratch,
                                 uint64_t scratch_bytes) {
  static const float kNoReward = 0.0f;  // not read by the dense pass
  return td_launch(ctx, n_features, fields, active_idx, active_val, n_active, &kNoReward,
                   globals, nullptr, scratch, scratch_bytes, kTdRunApply);
}
