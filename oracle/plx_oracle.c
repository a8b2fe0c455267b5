/*
 * plx_oracle.c — CPU restatement of the Plastix per-connection hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the sm_100a kernels:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * it. The product library (plastix_b200/libplastix_b200.so) never calls it.
 *
 * Every function restates one loop of the reference (paths relative to the
 * reference project) with the same evaluation order and single-precision
 * rounding: built with -O2 -ffp-contract=off on x86-64 (SSE, no FMA), as the
 * reference is. Parity of this restatement with the reference itself is pinned
 * by tests/test_oracle_pins.py against oracle/_ref (the reference headers
 * compiled by oracle/build.py) and the committed fixtures in tests/golden/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define APPLY_IDENTITY 0
#define APPLY_SIGMOID 1
#define APPLY_TANH 2
#define APPLY_IPC_ERROR 3

static float apply_value(int kind, float acc, float value) {
  switch (kind) {
    case APPLY_SIGMOID: /* examples/mlp-xor/mlp_xor.cpp:24-26 */
      return 1.0f / (1.0f + expf(-acc));
    case APPLY_TANH: /* examples/manual-fcc/manual_fcc.cpp Apply */
      return tanhf(acc);
    case APPLY_IPC_ERROR: /* examples/ipc-multilayer/ipc_multilayer.cpp:147-150 */
      return value - acc;
    default: /* include/plastix/traits.hpp:115-117 */
      return acc;
  }
}

/*
 * Network::DoForwardPass, Pipeline branch (include/plastix/plastix.hpp:133-148)
 * with DefaultForwardPass Map/Combine (traits.hpp:110-114):
 *   for C in connection order: skip Dead; Acc[To] = Acc[To] + W[C]*Act[From]
 *   for I in [num_input, n_units): Apply(Acc[I]); Acc[I] = 0
 * `act` is the whole Activation array; for IPC_ERROR the result goes to
 * err[I] (ErrorTag) and Activation is left alone, as in the iPC example.
 * fwd_acc must hold n_units zeros on entry (the reference resets it after
 * each Apply) and holds zeros again on return.
 */
void oracle_forward_pipeline(uint64_t n_conn, const uint32_t* from,
                             const uint32_t* to, const uint8_t* dead,
                             const float* w, float* act, uint64_t n_units,
                             uint64_t num_input, int apply_kind,
                             const float* value, float* err, float* fwd_acc) {
  for (uint64_t c = 0; c < n_conn; ++c) {
    if (dead && dead[c]) continue;
    fwd_acc[to[c]] = fwd_acc[to[c]] + w[c] * act[from[c]];
  }
  for (uint64_t i = num_input; i < n_units; ++i) {
    float v = apply_value(apply_kind, fwd_acc[i], value ? value[i] : 0.0f);
    if (apply_kind == APPLY_IPC_ERROR) err[i] = v;
    else act[i] = v;
    fwd_acc[i] = 0.0f;
  }
}

/*
 * DoUpdateConnectionState (plastix.hpp:238-245) with the per-connection
 * Hebbian trace rule used by the single-layer sweep workload:
 *   UpdateIncomingConnection: E = decay*E + Act[From]*Act[To]; W += rate*E
 */
void oracle_update_hebbian_trace(uint64_t n_conn, const uint32_t* from,
                                 const uint32_t* to, const uint8_t* dead,
                                 const float* act, float* w, float* trace,
                                 float decay, float rate) {
  for (uint64_t c = 0; c < n_conn; ++c) {
    if (dead && dead[c]) continue;
    trace[c] = decay * trace[c] + act[from[c]] * act[to[c]];
    w[c] += rate * trace[c];
  }
}

/*
 * DoUpdateConnectionState with the gradient rule of mlp_xor.cpp:51-56 and
 * linear_regression.cpp:31-36 (kind 1: W -= rate*Post[To]*Act[From]) or the
 * iPC Hebbian rule of ipc_multilayer.cpp:183-190 (kind 2:
 * W += rate*Post[To]*Act[From]). Post is a per-unit array.
 */
void oracle_update_post(uint64_t n_conn, const uint32_t* from,
                        const uint32_t* to, const uint8_t* dead,
                        const float* act, const float* post, int kind,
                        float rate, float* w) {
  for (uint64_t c = 0; c < n_conn; ++c) {
    if (dead && dead[c]) continue;
    if (kind == 1) w[c] -= rate * post[to[c]] * act[from[c]];
    else w[c] += rate * post[to[c]] * act[from[c]];
  }
}

/*
 * One sweep of the single-layer workload through DoStep in Pipeline mode:
 * DoForwardPass (identity Apply) followed by the Hebbian trace update.
 * act holds n_units entries; inputs are act[0, num_input).
 */
void oracle_step_hebbian(uint64_t n_conn, const uint32_t* from,
                         const uint32_t* to, const uint8_t* dead, float* w,
                         float* trace, float* act, uint64_t n_units,
                         uint64_t num_input, float decay, float rate,
                         float* fwd_acc) {
  oracle_forward_pipeline(n_conn, from, to, dead, w, act, n_units, num_input,
                          APPLY_IDENTITY, NULL, NULL, fwd_acc);
  oracle_update_hebbian_trace(n_conn, from, to, dead, act, w, trace, decay,
                              rate);
}

/* ---- permutation machinery (SOAAllocator::Gather, alloc.hpp:145-156) ---- */

/* dst[i] = src[perm[i]] for i < n, elements of `elem` bytes. */
void oracle_gather(const uint64_t* perm, uint64_t n, const void* src,
                   void* dst, uint32_t elem) {
  const unsigned char* s = (const unsigned char*)src;
  unsigned char* d = (unsigned char*)dst;
  for (uint64_t i = 0; i < n; ++i)
    memcpy(d + i * elem, s + perm[i] * elem, elem);
}

/*
 * Survivor permutation of DoPruneConnections' tombstones
 * (plastix.hpp:280-297 marks Dead; no compaction exists in the reference):
 * the increasing ids with keep[c] != 0. Returns the survivor count.
 */
uint64_t oracle_survivors(const uint8_t* keep, uint64_t n, uint64_t* perm) {
  uint64_t m = 0;
  for (uint64_t c = 0; c < n; ++c)
    if (keep[c]) perm[m++] = c;
  return m;
}

/*
 * Stable sort permutation by 32-bit key (counting sort on 16-bit halves,
 * LSD), the order std::stable_sort of ids by key produces. Used for the
 * re-sort by ToId and for SortConnectionsByLevel's stable counting sort by
 * SrcLevel (plastix.hpp:553-577).
 */
int oracle_stable_sort_u32(const uint32_t* key, uint64_t n, uint64_t* perm) {
  uint64_t* tmp = (uint64_t*)malloc((n ? n : 1) * sizeof(uint64_t));
  uint64_t* cnt = (uint64_t*)calloc(65537, sizeof(uint64_t));
  if (!tmp || !cnt) {
    free(tmp);
    free(cnt);
    return -1;
  }
  for (uint64_t i = 0; i < n; ++i) perm[i] = i;
  for (int pass = 0; pass < 2; ++pass) {
    const int sh = 16 * pass;
    memset(cnt, 0, 65537 * sizeof(uint64_t));
    for (uint64_t i = 0; i < n; ++i) cnt[((key[perm[i]] >> sh) & 0xFFFF) + 1]++;
    for (int b = 0; b < 65536; ++b) cnt[b + 1] += cnt[b];
    for (uint64_t i = 0; i < n; ++i) {
      uint32_t d = (key[perm[i]] >> sh) & 0xFFFF;
      tmp[cnt[d]++] = perm[i];
    }
    memcpy(perm, tmp, n * sizeof(uint64_t));
  }
  free(tmp);
  free(cnt);
  return 0;
}

/*
 * DoAddConnections phases 2-3 (plastix.hpp:411-432): sort the packed
 * CompactEdge bits (From | To<<32) ascending and keep the first of each run
 * of equal values. Sorts `bits` in place; returns the unique count written to
 * `out`.
 */
static int cmp_u64(const void* a, const void* b) {
  uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
  return x < y ? -1 : (x > y ? 1 : 0);
}

uint64_t oracle_sort_unique_u64(uint64_t* bits, uint64_t n, uint64_t* out) {
  qsort(bits, n, sizeof(uint64_t), cmp_u64);
  uint64_t m = 0, prev = UINT64_MAX;
  for (uint64_t i = 0; i < n; ++i) {
    if (bits[i] == prev) continue;
    prev = bits[i];
    out[m++] = bits[i];
  }
  return m;
}

/* ---- structural plasticity workload ------------------------------------ */

/* SplitMix64 finaliser (Steele, Lea, Flood 2014), the mixing function of the
 * seeded regrowth (same definition as the device generator). */
uint64_t oracle_mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* Connections [count, n) get fresh endpoints, weight 0, age 0. */
void oracle_regrow(uint64_t n, uint64_t count, uint32_t* from, uint32_t* to,
                   float* w, uint8_t* age, uint32_t src_base, uint32_t n_src,
                   uint32_t dst_base, uint32_t n_dst, uint64_t seed,
                   uint64_t step_base) {
  const uint64_t key = oracle_mix64(seed) + step_base;
  for (uint64_t i = count; i < n; ++i) {
    const uint64_t h = oracle_mix64(key + (i - count));
    from[i] = src_base + (uint32_t)(((h & 0xffffffffull) * n_src) >> 32);
    to[i] = dst_base + (uint32_t)(((h >> 32) * n_dst) >> 32);
    if (w) w[i] = 0.0f;
    if (age) age[i] = 0;
  }
}

/* The structural step's prune rule as a PruneConn policy would state it
 * (ShouldPrune = |w| < threshold, plastix.hpp:290-293): keep = !(|w| < thr). */
void oracle_keep_abs_ge(const float* w, uint64_t n, float thr, uint8_t* keep) {
  for (uint64_t c = 0; c < n; ++c) keep[c] = !(fabsf(w[c]) < thr);
}

/* ---- SwiftTD (examples/swifttd/swifttd.cpp:47-191) ---------------------- */

/* Globals of the SwiftTD network (swifttd.cpp:47-62): six hyperparameters,
 * then the seven running values. The device code uses the same layout. */
typedef struct {
  float gamma, lambda, eta, eta_min, decay, meta;
  float v, v_old, delta, v_delta_prev, v_delta, tau, b;
} oracle_td_globals;

/* One Network::DoStep of the SwiftTD network: N features (units 0..N-1) feed
 * one value unit over connections 0..N-1. fld[10] = W, Z, ZDelta, DeltaW, H,
 * HOld, HTemp, ZBar, P, Beta (swifttd.cpp:199-209 field order). The step is
 * DoForwardPass (V = W.F folded in connection order, Apply stores V,
 * swifttd.cpp:74-85), Loss (:90-100), the UpdateIncoming sweep over all
 * connections (phase 1, :106-150), the UpdateOutgoing sweep (phase 2,
 * :152-186) and ResetGlobal (:189-191); plastix.hpp:232-256 runs the two
 * sweeps in connection order.
 *
 * acc_f64 = 0 folds V, Tau, B and VDelta in fp32 in connection order, exactly
 * as the reference. acc_f64 = 1 folds the same fp32 terms in double and rounds
 * once: the parallel device reductions are compared against this form, since
 * a sequential fp32 sum over ~2e4 terms carries its own rounding error of
 * order 1e-5. Returns V. */
float oracle_swifttd_step(uint64_t n, float** fld, const float* f, float reward,
                          oracle_td_globals* g, int acc_f64) {
  float *W = fld[0], *Z = fld[1], *Zd = fld[2], *Dw = fld[3], *H = fld[4];
  float *HOld = fld[5], *HTemp = fld[6], *ZBar = fld[7], *P = fld[8], *Beta = fld[9];
  float acc = 0.0f;
  double acc_d = 0.0;
  for (uint64_t i = 0; i < n; ++i) {
    const float t = W[i] * f[i];
    acc = acc + t;
    acc_d += (double)t;
  }
  g->v = acc_f64 ? (float)acc_d : acc;
  g->delta = reward + g->gamma * g->v - g->v_old;
  g->v_delta_prev = g->v_delta;
  g->v_delta = 0.0f;
  g->tau = 0.0f;
  g->b = 0.0f;
  double tau_d = 0.0, b_d = 0.0, vd_d = 0.0;
  for (uint64_t i = 0; i < n; ++i) {
    const float F = f[i];
    Dw[i] = g->delta * Z[i] - Zd[i] * g->v_delta_prev;
    W[i] += Dw[i];
    Beta[i] += g->meta / expf(Beta[i]) * (g->delta - g->v_delta_prev) * P[i];
    float eb = expf(Beta[i]);
    if (eb > g->eta || isinf(eb)) {
      Beta[i] = logf(g->eta);
      eb = g->eta;
    }
    if (eb < g->eta_min) {
      Beta[i] = logf(g->eta_min);
      eb = g->eta_min;
    }
    HOld[i] = H[i];
    H[i] = HTemp[i] + g->delta * ZBar[i] - Zd[i] * g->v_delta_prev;
    HTemp[i] = H[i];
    Zd[i] = 0.0f;
    const float td = g->gamma * g->lambda;
    Z[i] *= td;
    P[i] *= td;
    ZBar[i] *= td;
    const float t_tau = eb * F * F, t_b = Z[i] * F;
    g->tau += t_tau;
    g->b += t_b;
    tau_d += (double)t_tau;
    b_d += (double)t_b;
  }
  if (acc_f64) {
    g->tau = (float)tau_d;
    g->b = (float)b_d;
  }
  for (uint64_t i = 0; i < n; ++i) {
    const float F = f[i];
    const float t_vd = Dw[i] * F;
    g->v_delta += t_vd;
    vd_d += (double)t_vd;
    float mult = 1.0f;
    if (g->tau > 0.0f && g->eta / g->tau < 1.0f) mult = g->eta / g->tau;
    Zd[i] = mult * expf(Beta[i]) * F;
    Z[i] += Zd[i] * (1.0f - g->b);
    P[i] += HOld[i] * F;
    ZBar[i] += Zd[i] * (1.0f - g->b - ZBar[i] * F);
    HTemp[i] = H[i] - HOld[i] * F * (Z[i] - Zd[i]) - H[i] * Zd[i] * F;
    if (g->tau > g->eta) {
      HTemp[i] = 0.0f;
      H[i] = 0.0f;
      HOld[i] = 0.0f;
      ZBar[i] = 0.0f;
      Beta[i] += logf(g->decay) * F * F;
    }
  }
  if (acc_f64) g->v_delta = (float)vd_d;
  g->v_old = g->v;
  return g->v;
}

/* ---- backward pass and per-unit steps of the example networks ----------- */

/* Backward Apply (kinds as the device: 0 store, 4 sigmoid gradient
 * mlp_xor.cpp:43-46, 5 iPC bottom-up ipc_multilayer.cpp:128-131,170-175). */
static float backward_apply(int kind, float acc, float value) {
  if (kind == 4) return acc * value * (1.0f - value);
  if (kind == 5) {
    const float t = tanhf(value);
    return (1.0f - t * t) * acc;
  }
  return acc;
}

/*
 * Network::DoBackwardPass over connections [0, n_conn) of the given arrays:
 * Pipeline order (descending = 1, plastix.hpp:193-203) or one Topological
 * level range (descending = 0, plastix.hpp:172-181). Map = W[C] * dval[To[C]]
 * (mlp_xor.cpp:38-41, ipc_multilayer.cpp:163-166), Combine = +. Then
 * out[I] = Apply(acc[I], value[I]) for I in [lo, hi) and acc is cleared for
 * all n_units units. bwd_acc holds n_units zeros on entry and on return.
 */
void oracle_backward(uint64_t n_conn, const uint32_t* from, const uint32_t* to,
                     const uint8_t* dead, const float* w, const float* dval,
                     int descending, uint64_t n_units, uint64_t lo, uint64_t hi,
                     int apply_kind, const float* value, float* out,
                     float* bwd_acc) {
  for (uint64_t j = 0; j < n_conn; ++j) {
    const uint64_t c = descending ? n_conn - 1 - j : j;
    if (dead && dead[c]) continue;
    bwd_acc[from[c]] = bwd_acc[from[c]] + w[c] * dval[to[c]];
  }
  for (uint64_t i = lo; i < hi; ++i)
    out[i] = backward_apply(apply_kind, bwd_acc[i], value ? value[i] : 0.0f);
  for (uint64_t i = 0; i < n_units; ++i) bwd_acc[i] = 0.0f;
}

/* iPC value-node update and pre-step (ipc_multilayer.cpp:239-245, :220-228),
 * as plx_ipc_value_update. */
void oracle_ipc_value_update(uint64_t n, float* x, const float* eps, float* bu,
                             float gamma, float* act, int mode) {
  for (uint64_t i = 0; i < n; ++i) {
    if (mode) {
      x[i] += gamma * (-eps[i] + bu[i]);
      bu[i] = 0.0f;
    }
    act[i] = tanhf(x[i]);
  }
}

/* MSELoss + sigmoid backward Apply of the outputs (traits.hpp:185-193,
 * mlp_xor.cpp:43-46). */
void oracle_mse_sigmoid_grad(uint64_t n, const float* act, const float* target,
                             float* grad) {
  for (uint64_t i = 0; i < n; ++i) {
    const float acc = act[i] - target[i];
    grad[i] = acc * act[i] * (1.0f - act[i]);
  }
}

/* RecomputeLevels (include/plastix/plastix.hpp:466-537), restated: levels of
 * the non-input units go to 0; nothing more without connections (:470-474).
 * Live connections give in-degrees by ToId and outgoing lists by FromId
 * (:488-512). Round L walks frontier L (round 0: the input units, :515-517);
 * every live outgoing connection of a frontier unit decrements its target's
 * in-degree (uint32, wrapping), and the decrement reaching 0 gives the target
 * level L+1 (uint16) and appends it to frontier L+1 (:519-535). Returns the
 * number of non-empty frontiers; -1 when a connection names a unit outside
 * [0, n_units) or memory runs out. */
int64_t oracle_recompute_levels(uint32_t n_units, uint32_t n_input, uint64_t n_conns,
                                const uint32_t* from, const uint32_t* to,
                                const uint8_t* dead, uint16_t* level) {
  for (uint32_t i = n_input; i < n_units; ++i) level[i] = 0;
  if (n_conns == 0) return 0;
  uint32_t* indeg = calloc((size_t)n_units + 1, sizeof(uint32_t));
  uint32_t* start = calloc((size_t)n_units + 2, sizeof(uint32_t));
  uint32_t* targets = malloc((n_conns ? n_conns : 1) * sizeof(uint32_t));
  uint32_t* cur = malloc(((size_t)n_units + 1) * sizeof(uint32_t));
  uint32_t* nxt = malloc(((size_t)n_units + 1) * sizeof(uint32_t));
  int64_t rounds = -1;
  if (!indeg || !start || !targets || !cur || !nxt) goto done;
  for (uint64_t c = 0; c < n_conns; ++c) {
    if (dead && dead[c]) continue;
    if (from[c] >= n_units || to[c] >= n_units) goto done;
    start[from[c] + 1]++;
    indeg[to[c]]++;
  }
  for (uint32_t i = 0; i < n_units; ++i) start[i + 1] += start[i];
  {
    /* outgoing lists in connection order: targets[start[u] .. start[u+1]) */
    uint32_t* fill = malloc(((size_t)n_units + 1) * sizeof(uint32_t));
    if (!fill) goto done;
    memcpy(fill, start, ((size_t)n_units + 1) * sizeof(uint32_t));
    for (uint64_t c = 0; c < n_conns; ++c) {
      if (dead && dead[c]) continue;
      targets[fill[from[c]]++] = to[c];
    }
    free(fill);
  }
  uint32_t n_cur = n_input;
  for (uint32_t i = 0; i < n_input; ++i) cur[i] = i;
  rounds = 0;
  for (uint32_t L = 0; n_cur > 0; ++L) {
    uint32_t n_nxt = 0;
    for (uint32_t f = 0; f < n_cur; ++f) {
      const uint32_t u = cur[f];
      for (uint32_t e = start[u]; e < start[u + 1]; ++e) {
        const uint32_t t = targets[e];
        indeg[t] -= 1u;
        if (indeg[t] == 0) {
          level[t] = (uint16_t)(L + 1u);
          nxt[n_nxt++] = t;
        }
      }
    }
    uint32_t* sw = cur;
    cur = nxt;
    nxt = sw;
    n_cur = n_nxt;
    ++rounds;
  }
done:
  free(indeg);
  free(start);
  free(targets);
  free(cur);
  free(nxt);
  return rounds;
}
