/*
 * plastix_b200.h — C ABI of the B200 (sm_100a) per-connection hot path.
 *
 * Every entry point takes plain device pointers and sizes, enqueues its
 * kernels on the context's stream and returns a status code (PLX_OK = 0).
 * Nothing here synchronises the stream except plx_ctx_sync().
 * The failing call's message is available from plx_last_error() on the same
 * host thread.
 *
 * Data layout (the reference's SoA field arrays, reference
 * include/plastix/conn.hpp:31-36 and include/plastix/unit_state.hpp:38-44,
 * mirrored into device memory):
 *   connection fields  FromId u32, ToId u32, Dead u8 (bool), Weight f32, ...
 *                      one array per field, indexed by connection id;
 *   unit fields        Activation f32, ...   one array per field.
 * The sweeps require the connections to be sorted by ToId (stable). The
 * reference accumulates ForwardAcc[ToId] in connection-index order
 * (include/plastix/plastix.hpp:133-141); a stable dst sort keeps that order
 * inside each destination, so the per-destination sums reproduce the
 * reference bit for bit for rows of up to PLX_SEQ_ROW_MAX connections.
 */
#ifndef PLASTIX_B200_H
#define PLASTIX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define PLX_OK 0
#define PLX_ERR_ARG 1         /* invalid argument (null, misaligned, size)  */
#define PLX_ERR_CUDA 2        /* CUDA runtime error                          */
#define PLX_ERR_CAPACITY 3    /* size exceeds a documented maximum           */
#define PLX_ERR_TIMEOUT 4     /* a bounded device-side wait expired          */
#define PLX_ERR_UNSUPPORTED 5 /* option not implemented                      */

/* Rows (destination units) with at most this many connections are summed
 * strictly left to right, exactly like the reference loop. Longer rows use a
 * fixed deterministic order: 32 lane-strided partial sums (every 32nd
 * connection) folded in lane order; rows over 8192 connections use 256
 * thread-strided partial sums. */
#define PLX_SEQ_ROW_MAX 256

/* ---- library / context ------------------------------------------------- */

/* Replaces plastix::version() (reference src/plastix.cpp:5): "0.1.0". */
const char* plx_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* plx_last_error(void);

typedef struct plx_ctx plx_ctx;

/* Creates a context on `device` that enqueues on `stream` (a cudaStream_t;
 * NULL = the legacy default stream). Allocates one device status word. */
int plx_ctx_create(int device, void* stream, plx_ctx** out);
int plx_ctx_destroy(plx_ctx* ctx);
int plx_ctx_set_stream(plx_ctx* ctx, void* stream);
/* Wall-clock limit of every bounded device-side wait (default 2 s). */
int plx_ctx_set_timeout_ns(plx_ctx* ctx, uint64_t timeout_ns);
int plx_ctx_num_sms(plx_ctx* ctx, int* out);
/* Waits for the stream, then reads and clears the device status word:
 * PLX_ERR_TIMEOUT if a bounded wait expired since the last sync. */
int plx_ctx_sync(plx_ctx* ctx);

/* ---- CSR view of dst-sorted connections -------------------------------- */

/* row_ptr[r] = first connection whose ToId >= row_base + r, r in [0,n_rows]
 * (row_ptr[n_rows] = n_edges); to_id must be sorted ascending, 16-byte
 * aligned. One pass over the connections. Derived index over the reference's
 * ToId field (conn.hpp:13). */
int plx_csr_row_ptr(plx_ctx* ctx, const uint32_t* to_id, uint64_t n_edges,
                    uint32_t row_base, uint32_t n_rows, uint32_t* row_ptr);

typedef struct plx_csr {
  const uint32_t* row_ptr; /* n_rows + 1 entries, row_ptr[0] == 0          */
  const uint32_t* plan;    /* from plx_csr_plan                             */
  const uint32_t* to_id;   /* optional ToId field (see below), or NULL      */
  uint64_t n_edges;        /* == row_ptr[n_rows], < 2^32 - 2^16             */
  uint32_t n_rows;
  uint32_t row_base;       /* unit id of row 0 (ToId of its connections)    */
  uint32_t n_wide;         /* rows with PLX_SEQ_ROW_MAX < length <= 8192    */
  uint32_t n_long;         /* rows longer than 8192                         */
  uint32_t n_short;        /* rows of at most PLX_SEQ_ROW_MAX (incl. empty) */
  uint32_t max_row;        /* connections in the longest row                */
} plx_csr;
/* plx_csr_plan fills every member except to_id (set to NULL) and row_base
 * (set to 0). When the caller sets to_id (the dst-sorted ToId field, 16-byte
 * aligned, consistent with row_ptr) and row_base, sweeps over CSRs whose rows
 * all have at most PLX_SEQ_ROW_MAX connections run the register-resident
 * warp kernel; otherwise the tile kernel. Results are identical. */

/* Size (in u32 words) of the sweep plan for n_edges connections. */
uint64_t plx_csr_plan_words(uint64_t n_edges, uint32_t n_rows);

/* Validates row_ptr, classifies the rows (short / wide / long) and builds the
 * tile plan every sweep over this row_ptr uses. Fills *out (row_ptr, plan,
 * sizes and row counts). row_ptr must be 16-byte aligned. Synchronises the
 * stream. The plan stays valid while row_ptr is unchanged. */
int plx_csr_plan(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                 uint64_t n_edges, uint32_t* plan, uint64_t plan_words,
                 plx_csr* out);

/* Same as plx_csr_plan without synchronising: out's row counts are set to
 * PLX_COUNT_UNKNOWN and the sweeps then read them on the device (launching
 * the wide/long-row kernels unconditionally). An invalid row_ptr is reported
 * by plx_ctx_sync (PLX_ERR_ARG) after the sweep. For per-step re-planning. */
int plx_csr_plan_async(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                       uint64_t n_edges, uint32_t* plan, uint64_t plan_words,
                       plx_csr* out);

#define PLX_COUNT_UNKNOWN 0xFFFFFFFFu

/* ---- forward sweep (Map / Combine / Apply) ----------------------------- */

/* Apply kinds (the unit-side policy run once per destination row). */
#define PLX_APPLY_IDENTITY 0  /* act = acc            traits.hpp:115-117   */
#define PLX_APPLY_SIGMOID 1   /* act = 1/(1+exp(-acc))  mlp_xor.cpp:24-26  */
#define PLX_APPLY_TANH 2      /* act = tanh(acc)      manual_fcc Apply      */
#define PLX_APPLY_IPC_ERROR 3 /* err = x - acc        ipc_multilayer.cpp:147-150 */
/* Backward-pass applies (the sweep run over a source-major connection order,
 * see plx_transpose): value[r] is the row unit's activation or value node. */
#define PLX_APPLY_SIGMOID_GRAD 4 /* out = acc * a * (1 - a)   mlp_xor.cpp:43-46 */
#define PLX_APPLY_TANH_GRAD 5    /* out = (1 - tanh(x)^2) * acc
                                    ipc_multilayer.cpp:128-131,170-175        */

/* One forward sweep with the default Map/Combine (w * act[src], +), then
 * Apply per row. Replaces Network::DoForwardPass, Pipeline branch
 * (plastix.hpp:133-148) and one level of the Topological branch
 * (plastix.hpp:112-130) for a contiguous range of destination units.
 *   from_id   [n_edges]  FromId field (absolute unit ids)
 *   weight    [n_edges]  Weight field
 *   dead      [n_edges]  Dead field, or NULL when no connection is dead
 *   act_src              Activation array indexed by FromId, act_src_len
 *                        entries (an out-of-range FromId reads 0 and makes
 *                        plx_ctx_sync report PLX_ERR_ARG)
 *   act_dst   [n_rows]   Activation of the rows (written; not for IPC_ERROR)
 *   value     [n_rows]   IPC_ERROR only: value-node x of each row (read)
 *   err_out   [n_rows]   IPC_ERROR only: eps = x - acc (written)
 * Connection arrays must be 16-byte aligned. */
int plx_sweep_forward(plx_ctx* ctx, const plx_csr* csr, const uint32_t* from_id,
                      const float* weight, const uint8_t* dead,
                      const float* act_src, uint32_t act_src_len,
                      int apply_kind, float* act_dst, const float* value,
                      float* err_out);

/* plx_sweep_forward over a CSR given by row_ptr alone (no plan), one thread
 * per row folding its connections left to right -- the reference's order
 * for every row length, so row values equal the reference's bit for bit.
 * For layers of a few connections per row (the structural workload: two
 * per destination), where it is the faster sweep and spares the plan.
 * act_src_len bounds the gathered ids (an id past it reads 0 and sets the
 * status word). */
int plx_sweep_forward_rows(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows,
                           const uint32_t* from_id, const float* weight, const uint8_t* dead,
                           const float* act_src, uint32_t act_src_len, int apply_kind,
                           float* act_dst, const float* value, float* err_out);

/* Forward sweep fused with the per-connection Hebbian trace rule
 *   acc = sum w*act[src];  post = acc (identity Apply);
 *   trace' = decay*trace + act[src]*post;  w' = w + rate*trace'
 * in one pass over the connection SoA. Replaces DoForwardPass followed by
 * DoUpdateConnectionState (plastix.hpp:133-148, :238-245) for that rule.
 * Reads w_in/trace_in and writes w_out/trace_out (distinct buffers; the sweep
 * re-reads neighbouring rows' old weights). act_dst receives post. */
int plx_sweep_forward_hebbian(plx_ctx* ctx, const plx_csr* csr,
                              const uint32_t* from_id, const uint8_t* dead,
                              const float* act_src, uint32_t act_src_len,
                              const float* w_in, float* w_out,
                              const float* trace_in,
                              float* trace_out, float decay, float rate,
                              float* act_dst);

/* ---- warp-sliced row layout (the fused sweep, one lane per row) ---------- */

#define PLX_SLICED_NONE 0xFFFFFFFFu

/* Connections of a destination-sorted CSR re-laid for a sweep in which one
 * lane owns one row: rows are taken in windows of 512 consecutive rows,
 * ordered by length inside each window (descending, stable) and dealt 32 at
 * a time into slices. Slot slice_ptr[s] + 128*g + 4*l + c holds connection
 * 4g + c of the row of lane l of slice s; shorter rows leave padding slots.
 * Every connection field of a sliced layer is stored in slot order;
 * perm[slot] is the slot's reference connection index (PLX_SLICED_NONE for
 * padding). All arrays are device memory. */
typedef struct plx_sliced {
  const uint64_t* slice_ptr; /* [n_slices + 1] first slot of each slice       */
  const uint32_t* lane_row;  /* [n_slices * 32] row of each lane (or NONE)    */
  const uint32_t* lane_len;  /* [n_slices * 32] connections of that row       */
  const uint32_t* perm;      /* [n_slots] reference index of each slot        */
  uint64_t n_slots;
  uint64_t n_edges;
  uint32_t n_rows;
  uint32_t n_slices; /* ceil(n_rows / 32) */
} plx_sliced;

uint32_t plx_sliced_n_slices(uint32_t n_rows);
size_t plx_sliced_plan_scratch_bytes(uint32_t n_rows);

/* Builds the slices of a CSR (row_ptr as from plx_csr_row_ptr) into the
 * caller's arrays (slice_ptr: n_slices + 1 u64, lane_row / lane_len:
 * n_slices * 32 u32) and fills *out, including n_slots (this call waits for
 * the stream to read it back; allocate the slot arrays from it). perm is
 * left NULL until plx_sliced_perm. Replaces nothing in the reference: it is
 * the storage order of the sweep below. */
int plx_sliced_plan(plx_ctx* ctx, const uint32_t* row_ptr, uint32_t n_rows, uint64_t n_edges,
                    plx_sliced* out, uint64_t* slice_ptr, uint32_t* lane_row,
                    uint32_t* lane_len, void* scratch, size_t scratch_bytes);
/* perm[slot] (n_slots u32, 16-byte aligned) from the CSR; sets out->perm. */
int plx_sliced_perm(plx_ctx* ctx, plx_sliced* sl, const uint32_t* row_ptr, uint32_t* perm);
/* slot[i] = ref[perm[i]] (zero for padding) / ref[perm[i]] = slot[i], for
 * one field of 1, 2, 4 or 8 bytes per element. */
int plx_sliced_pack(plx_ctx* ctx, const plx_sliced* sl, const void* ref, void* slot,
                    uint32_t elem_bytes);
int plx_sliced_unpack(plx_ctx* ctx, const plx_sliced* sl, const void* slot, void* ref,
                      uint32_t elem_bytes);

/* plx_sweep_forward_hebbian (DoForwardPass, Pipeline, identity Apply, then
 * the trace rule of DoUpdateConnectionState, plastix.hpp:133-148 and
 * :238-245) over a sliced layer: from_id, dead (optional), weight and trace
 * in slot order; weight and trace are updated in place. Every row is folded
 * left to right by one lane, so row values, weights and traces equal the
 * reference's bit for bit, whatever the row lengths. act_dst is indexed by
 * row. With n_peers > 0 each row value is also stored to
 * peer_out[p][peer_offset + r], as plx_sweep_forward_hebbian_gather (same
 * peer_len check). */
int plx_sweep_forward_hebbian_sliced(plx_ctx* ctx, const plx_sliced* sl, const uint32_t* from_id,
                                     const uint8_t* dead, const float* act_src,
                                     uint32_t act_src_len, float* weight, float* trace,
                                     float decay, float rate, float* act_dst,
                                     float* const* peer_out, uint32_t n_peers,
                                     uint32_t peer_offset, uint32_t peer_len);

/* ---- hand-off over peer memory (one process per GPU, NVLink) ------------ */

#define PLX_MAX_PEERS 8
#define PLX_IPC_HANDLE_BYTES 64

/* The fused sweep of plx_sweep_forward_hebbian that also hands the layer's
 * output to the other GPUs: every destination value is stored, besides
 * act_dst, to peer_out[p][peer_offset + r] for each of the n_peers buffers
 * (the all-gather buffers of every GPU, this one's included, mapped with
 * plx_peer_open), so the all-gather of destination slices after a sweep
 * (the multi-GPU hand-off between layers) rides on the sweep's own stores
 * over NVLink. Follow it with plx_peer_barrier before reading the buffer.
 * peer_len is the length (floats) of every peer buffer: the call fails with
 * PLX_ERR_ARG, before touching any device, unless
 * peer_offset + csr->n_rows <= peer_len, so a wrong offset or shard size can
 * never store past the end of another GPU's buffer. */
int plx_sweep_forward_hebbian_gather(
    plx_ctx* ctx, const plx_csr* csr, const uint32_t* from_id, const uint8_t* dead,
    const float* act_src, uint32_t act_src_len, const float* w_in, float* w_out,
    const float* trace_in, float* trace_out, float decay, float rate, float* act_dst,
    float* const* peer_out, uint32_t n_peers, uint32_t peer_offset, uint32_t peer_len);

/* Device memory another process can map: cudaMalloc'd and zeroed, its IPC
 * handle (PLX_IPC_HANDLE_BYTES bytes) written to ipc_handle. */
int plx_peer_alloc(plx_ctx* ctx, size_t bytes, void** ptr, void* ipc_handle);
int plx_peer_free(plx_ctx* ctx, void* ptr);
/* Maps a peer's allocation into this process (peer access enabled). */
int plx_peer_open(plx_ctx* ctx, const void* ipc_handle, void** ptr);
int plx_peer_close(plx_ctx* ctx, void* ptr);

/* Barrier over n GPUs: flags[p] is rank p's array of n uint64 counters
 * (peer memory). Publishes epoch (increasing per call) to every rank after a
 * system-scope fence over this GPU's earlier stores, then waits until every
 * rank published it. A wait beyond the context's timeout records
 * PLX_ERR_TIMEOUT (plx_ctx_sync) and returns; nothing blocks forever. */
int plx_peer_barrier(plx_ctx* ctx, uint64_t* const* flags, uint32_t n, uint32_t rank,
                     uint64_t epoch);

/* Device-to-device copy on the context's stream (e.g. out of a peer buffer). */
int plx_copy_device(plx_ctx* ctx, void* dst, const void* src, size_t bytes);

/* Unit levels: RecomputeLevels (include/plastix/plastix.hpp:466-537), the
 * level-parallel Kahn pass over live connections. Resets level[i] = 0 for
 * non-input units i in [n_input, n_units); then, from the input units as round
 * 0's frontier, each round decrements the in-degree of every live outgoing
 * target of the frontier, and a target whose in-degree reaches 0 in round L
 * gets level L+1 (uint16) and joins the next frontier. Bit-identical levels
 * to the reference (they do not depend on the order within a round).
 * *rounds_out (device, optional) receives the number of non-empty frontiers.
 * dead may be NULL (all live). Connections naming a unit >= n_units are
 * skipped and recorded as PLX_ERR_ARG at plx_ctx_sync. Runs one cooperative
 * kernel for all rounds; a grid barrier that waits past the context's
 * timeout records PLX_ERR_TIMEOUT. */
size_t plx_recompute_levels_scratch_bytes(uint64_t n_units, uint64_t n_conns);
int plx_recompute_levels(plx_ctx* ctx, uint32_t n_units, uint32_t n_input, uint64_t n_conns,
                         const uint32_t* from_id, const uint32_t* to_id, const uint8_t* dead,
                         uint16_t* level, uint32_t* rounds_out, void* scratch,
                         size_t scratch_bytes);

/* src_level[c] = level[from_id[c]]: the SrcLevel refresh of
 * SortConnectionsByLevel (plastix.hpp:546-549). Followed by
 * plx_radix_sort_u32 on the 16-bit key and plx_gather, it is the whole
 * re-sort (:551-577). */
int plx_src_levels(plx_ctx* ctx, uint64_t n_conns, const uint32_t* from_id,
                   const uint16_t* level, uint32_t n_units, uint16_t* src_level);

/* Update kinds for plx_sweep_update (per-connection, reads a per-row value). */
#define PLX_UPDATE_GRADIENT 1 /* w -= rate * post[dst] * act[src]
                                 (mlp_xor.cpp:51-56, linear_regression.cpp:31-36) */
#define PLX_UPDATE_HEBBIAN 2  /* w += rate * post[dst] * act[src]
                                 (ipc_multilayer.cpp:182-190)                 */
#define PLX_UPDATE_HEBBIAN_T 3 /* the same rule on a source-major copy, where
                                  the row value is act[src] and the gathered
                                  value post[dst]: w += (rate * post) * act,
                                  rounded in the same order as kind 2, so a
                                  source-major copy stays bit-identical */

/* Per-connection weight update over dst-sorted connections; replaces the
 * UpdateIncomingConnection sweep of DoUpdateConnectionState
 * (plastix.hpp:238-245) for the two rules above. post is indexed by row.
 * w_out may equal w_in. */
int plx_sweep_update(plx_ctx* ctx, const plx_csr* csr, const uint32_t* from_id,
                     const uint8_t* dead, const float* act_src,
                     uint32_t act_src_len, const float* post, int update_kind,
                     float rate, const float* w_in, float* w_out);

/* ---- structural change: compaction, re-sort, regrowth ------------------ */

#define PLX_MAX_FIELDS 16

/* One SoA field to move: element i of src goes to some position of dst. */
typedef struct plx_field {
  const void* src;
  void* dst;            /* must not overlap src                              */
  uint32_t elem_bytes;  /* 1, 2, 4 or 8                                      */
  uint32_t flags;       /* PLX_FIELD_*                                       */
} plx_field;

/* u8 field: the survivor's value is incremented, saturating at 255 (a
 * connection age counter). plx_compact only. */
#define PLX_FIELD_INC_SAT_U8 1u

/* Keep predicates of plx_compact. */
#define PLX_KEEP_FLAGS 0    /* keep_src u8: keep where != 0                     */
#define PLX_KEEP_NOT_DEAD 1 /* keep_src u8 (the Dead field): keep where == 0    */
#define PLX_KEEP_ABS_GE 2   /* keep_src f32: prune where |v| < threshold        */

size_t plx_compact_scratch_bytes(uint64_t n);

/* Order-preserving compaction of n connections (single-pass decoupled
 * lookback). Survivor j of every field lands at dst[j]; *count_out (DEVICE
 * memory) receives the survivor count; perm_out (optional, device) receives
 * the surviving ids. Equals the reference's SOAAllocator::Gather
 * (alloc.hpp:145-156) with the increasing list of ids that
 * DoPruneConnections (plastix.hpp:280-297) left alive. scratch: device memory
 * of plx_compact_scratch_bytes(n). */
int plx_compact(plx_ctx* ctx, uint64_t n, int keep_kind, const void* keep_src,
                float threshold, const plx_field* fields, uint32_t n_fields,
                uint32_t* perm_out, uint64_t* count_out, void* scratch,
                size_t scratch_bytes);

/* Same compaction, allocating nothing. No counterpart in the reference: it
 * exists for callers that cannot allocate device memory when they compact
 * (a step loop with a fixed memory budget, a host framework that owns all
 * device memory and forbids libraries from calling cudaMalloc). Neither the
 * caller nor the library allocates: the scratch is a static device array of
 * 512 KiB + 256 B that every GPU loading this library holds until exit.
 *   - n <= 2^28 connections (268,435,456); larger n returns PLX_ERR_ARG.
 *   - Runs on `stream` (a cudaStream_t) of the current device; no context.
 *   - The first call on a device looks up the array's device address; make
 *     that first call before any stream capture on the device.
 *   - Every call on a device shares the array. Calls whose kernels overlap
 *     on the GPU (different streams, no ordering between them) race and give
 *     wrong results: order them on one stream or with events.
 *   - If a bounded device-side wait expires, *count_out is set to UINT64_MAX.
 * Output and arguments are otherwise those of plx_compact. */
int plx_compact_noalloc(void* stream, uint64_t n, int keep_kind,
                        const void* keep_src, float threshold,
                        const plx_field* fields, uint32_t n_fields,
                        uint32_t* perm_out, uint64_t* count_out);

/* dst[i] = src[perm[i]] for i < n and every field: the reference's
 * SOAAllocator::Gather (alloc.hpp:145-156) on the device. */
int plx_gather(plx_ctx* ctx, uint64_t n, const uint32_t* perm,
               const plx_field* fields, uint32_t n_fields);

size_t plx_radix_sort_scratch_bytes(uint64_t n);

/* Stable LSD radix sort of n u32 keys on bits [begin_bit, end_bit): writes the
 * sorted keys and the sorting permutation (perm_out[i] = original index of
 * the i-th key). Replaces std::sort by CompactEdge bits (plastix.hpp:411-415)
 * and the stable counting sort by SrcLevel (plastix.hpp:553-577) for the
 * re-sort of connections by ToId. n < 2^30. */
int plx_radix_sort_u32(plx_ctx* ctx, uint64_t n, const uint32_t* keys_in,
                       uint32_t* keys_out, uint32_t* perm_out,
                       uint32_t begin_bit, uint32_t end_bit, void* scratch,
                       size_t scratch_bytes);

size_t plx_sort_tail_scratch_bytes(uint64_t n);

/* plx_radix_sort_u32 for keys whose first *n_sorted entries are already in
 * order (by bits [begin_bit, end_bit)) -- the connections a compaction kept,
 * followed by regrown ones: the tail is radix-sorted and merged with the
 * prefix (prefix first on equal keys). keys_out and perm_out equal
 * plx_radix_sort_u32's bit for bit when the precondition holds. n_sorted is
 * in DEVICE memory (plx_compact's count); this call waits for the stream to
 * read it. keys_out and perm_out 16-byte aligned; n < 2^30. Replaces, for
 * the re-sort after regrowth, the full sort of the reference's
 * Gather-by-sorted-order (alloc.hpp:145-156). */
int plx_sort_tail_u32(plx_ctx* ctx, uint64_t n, const uint64_t* n_sorted, const uint32_t* keys_in,
                      uint32_t* keys_out, uint32_t* perm_out, uint32_t begin_bit,
                      uint32_t end_bit, void* scratch, size_t scratch_bytes);

size_t plx_sort_unique_u64_scratch_bytes(uint64_t n);

/* Proposal commit of DoAddConnections (plastix.hpp:411-433): sorts n 64-bit
 * keys ((To << 32) | From, CompactEdge::Bits) ascending and writes each
 * distinct key once to out (the reference's std::sort + skip of repeats);
 * *count_out (DEVICE memory) receives the number written. n < 2^30. */
int plx_sort_unique_u64(plx_ctx* ctx, uint64_t n, const uint64_t* keys, uint64_t* out,
                        uint64_t* count_out, void* scratch, size_t scratch_bytes);

/* Regrowth after compaction: connections [*count, n) (count in DEVICE
 * memory) get FromId/ToId from a seeded counter-based generator, Weight 0
 * and age 0 (weight/age may be NULL). For the i-th regrown connection:
 *   h = mix64(mix64(seed) + step_base + i), mix64 = SplitMix64 finaliser;
 *   FromId = src_base + ((h & 0xffffffff) * n_src >> 32);
 *   ToId   = dst_base + ((h >> 32) * n_dst >> 32). */
int plx_regrow(plx_ctx* ctx, uint64_t n, const uint64_t* count,
               uint32_t* from_id, uint32_t* to_id, float* weight, uint8_t* age,
               uint32_t src_base, uint32_t n_src, uint32_t dst_base,
               uint32_t n_dst, uint64_t seed, uint64_t step_base);

/* ---- backward order and per-unit steps ----------------------------------- */

size_t plx_transpose_scratch_bytes(uint64_t n);

/* Source-major order of n connections for the backward sweep: a stable sort
 * by FromId (sources src_base .. src_base + n_src - 1; connections from other
 * units sort after them and belong to no row), each source's run in
 * DESCENDING connection index order when `reverse` is set -- the Pipeline
 * backward order, plastix.hpp:193-203 -- or ascending (the Topological level
 * sweep, plastix.hpp:172-181). Outputs: keys_out[j] = FromId - src_base of
 * position j (n_src for excluded connections), perm_out[j] = its connection
 * index (apply with plx_gather to ToId, Weight, ...), row_ptr_out[0..n_src].
 * A sweep over (row_ptr_out, gathered ToId as the gathered index, gathered
 * Weight) with a PLX_APPLY_*_GRAD apply is the reference's DoBackwardPass.
 * n < 2^30. */
int plx_transpose(plx_ctx* ctx, uint64_t n, const uint32_t* from_id,
                  uint32_t src_base, uint32_t n_src, int reverse,
                  uint32_t* keys_out, uint32_t* perm_out, uint32_t* row_ptr_out,
                  void* scratch, size_t scratch_bytes);

/* iPC value nodes of n hidden units (ipc_multilayer.cpp:239-245 then the
 * pre-step of the next step, :220-228): mode 1: x += gamma * (-eps + bu);
 * bu = 0; act = tanh(x). mode 0: act = tanh(x) only. */
int plx_ipc_value_update(plx_ctx* ctx, uint64_t n, float* x, const float* eps,
                         float* bu, float gamma, float* act, int mode);

/* MSELoss (traits.hpp:185-193) and the sigmoid backward Apply of the output
 * units (mlp_xor.cpp:43-46): grad = ((a - target) * a) * (1 - a). */
int plx_mse_sigmoid_grad(plx_ctx* ctx, uint64_t n, const float* act,
                         const float* target, float* grad);

/* ---- chunked-source layout for long rows --------------------------------- */

/* Sources per chunk: a chunk of gathered values (64 KB) sits in one CTA's
 * shared memory while it folds the chunk's share of many rows. */
#define PLX_CHUNK_SOURCES 16384

/* Connections of a row set stored by (chunk of the gathered side, row), each
 * (chunk, row) segment padded to a multiple of 4 connections; src holds the
 * 16-bit offset within the chunk (PLX_CHUNK_SOURCES marks padding, which
 * reads 0), perm the original connection index (0xFFFFFFFF for padding).
 * n_chunks = ceil(n_src / PLX_CHUNK_SOURCES). For rows of hundreds or
 * thousands of connections (the 2,048-fan-in multilayer network), where
 * global-memory gathers, not HBM, bound a CSR sweep. */
typedef struct plx_chunked {
  const uint32_t* seg_ptr; /* [n_chunks * n_rows + 1], chunk-major          */
  const uint16_t* src;     /* [n_padded]                                     */
  const uint32_t* perm;    /* [n_padded]                                     */
  uint32_t n_rows;
  uint32_t n_src;          /* gathered values per sweep                      */
  uint32_t n_chunks;
} plx_chunked;

/* Upper bound of the padded length (allocate src/perm/weights with it). */
uint64_t plx_chunked_max_padded(uint64_t n_edges, uint32_t n_rows, uint32_t n_src);
size_t plx_chunked_scratch_bytes(uint64_t n_edges, uint32_t n_rows, uint32_t n_src);

/* Builds the layout of n_edges connections whose gathered unit is gather_id
 * (units [src_base, src_base + n_src)) and whose row unit is row_id (units
 * [row_base, row_base + n_rows)); connections outside either range are left
 * out. Within a segment connections keep their index order. Forward sweep:
 * gather_id = FromId, row_id = ToId; backward: gather_id = ToId,
 * row_id = FromId. n_edges < 2^30 per call. */
int plx_chunked_build(plx_ctx* ctx, uint64_t n_edges, const uint32_t* gather_id,
                      uint32_t src_base, uint32_t n_src, const uint32_t* row_id,
                      uint32_t row_base, uint32_t n_rows, uint32_t* seg_ptr,
                      uint16_t* src, uint32_t* perm, void* scratch,
                      size_t scratch_bytes);

/* out[d] = field[perm[d]] (0 for padding): a connection field in layout order. */
int plx_chunked_gather(plx_ctx* ctx, uint64_t n_padded, const uint32_t* perm,
                       const float* field, float* out);

/* Row sweep over the layout: acc[r] = sum over the row's connections of
 * w * gathered[src] -- per chunk a lane-strided sum, chunks added in order
 * (deterministic; not the reference's left fold) -- then the apply rule:
 * out[r] = Apply(acc[r], value[r]). partial: n_chunks * n_rows floats. */
int plx_chunked_fold(plx_ctx* ctx, const plx_chunked* layout, const float* w,
                     const float* gathered, int apply_kind, const float* value,
                     float* out, float* partial);

/* plx_chunked_fold of an iPC backward block (apply TANH_GRAD, value = x)
 * with the value-node update of the same hidden units fused into its
 * epilogue -- plx_ipc_value_update mode 1 (ipc_multilayer.cpp:239-245 and
 * the pre-step :220-228): bu = (1 - tanh(x)^2) * acc; x += gamma * (-eps + bu);
 * act = tanh(x). The bottom-up sum itself is not stored (the reference
 * zeroes it after the update). x and act equal those of the two separate
 * calls bit for bit. Valid where nothing reads x or act between the backward
 * fold and the value update (an inference iteration; not the example's
 * learning step, whose connection update reads act in between). */
int plx_chunked_fold_ipc_value(plx_ctx* ctx, const plx_chunked* layout, const float* w,
                               const float* gathered, float* x, const float* eps, float gamma,
                               float* act, float* partial);

/* Per-connection update over the layout with row_val[r] as the row value and
 * gathered[src] as the other side, PLX_UPDATE_* rules with the rounding of
 * plx_sweep_update (a weight updated here equals the same rule applied to the
 * destination-major copy, bit for bit). Padding stays 0. */
int plx_chunked_update(plx_ctx* ctx, const plx_chunked* layout, float* w,
                       const float* gathered, const float* row_val, int update_kind,
                       float rate);

/* ---- SwiftTD (examples/swifttd/swifttd.cpp) ------------------------------ */

/* Number of per-feature SoA fields, in the reference's ExtraConnFields order
 * (swifttd.cpp:199-209): W, Z, ZDelta, DeltaW, H, HOld, HTemp, ZBar, P, Beta. */
#define PLX_TD_NUM_FIELDS 10

/* The network's globals (swifttd.cpp:47-62), in DEVICE memory: the six
 * hyperparameters (the caller sets them; the reference fixes them as member
 * initialisers) and the seven running values (start at zero). */
typedef struct plx_td_globals {
  float gamma, lambda, eta, eta_min, decay, meta;
  float v, v_old, delta, v_delta_prev, v_delta, tau, b;
} plx_td_globals;

/* Scratch for plx_swifttd_step with up to max_active active features. */
uint64_t plx_swifttd_scratch_bytes(uint64_t n_features, uint32_t max_active);

/* One Network::DoStep of the SwiftTD network (plastix.hpp:439-455 with the
 * swifttd.cpp policies): DoForwardPass (V = sum W*F, swifttd.cpp:74-85), Loss
 * (:90-100), the UpdateIncoming sweep (phase 1, :106-150), the UpdateOutgoing
 * sweep (phase 2, :152-186), ResetGlobal (:189-191).
 *   fields:     host array of PLX_TD_NUM_FIELDS device pointers, n_features
 *               floats each, 16-byte aligned; updated in place.
 *   active_idx: the features with F != 0, strictly increasing, < n_features
 *               (an unsorted or out-of-range list is reported by
 *               plx_ctx_sync as PLX_ERR_ARG); active_val their values, or
 *               NULL for binary features (all 1.0). Inactive features have
 *               F = 0 and still take the full update, as in the reference.
 *   reward:     DEVICE pointer to this step's reward (Targets[0]).
 *   v_out:      optional DEVICE pointer receiving V (GetOutput()[0]).
 *   scratch:    plx_swifttd_scratch_bytes(n_features, >= n_active) bytes,
 *               zero-filled before the first step; each step leaves it ready
 *               for the next.
 * V, Tau, B and VDelta are summed in double precision in a fixed order
 * (deterministic); the reference sums them sequentially in float. */
int plx_swifttd_step(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                     const uint32_t* active_idx, const float* active_val,
                     uint32_t n_active, const float* reward,
                     plx_td_globals* globals, float* v_out, void* scratch,
                     uint64_t scratch_bytes);

/* The two halves of plx_swifttd_step, for callers that time or schedule
 * them apart: plx_swifttd_reduce is DoForwardPass + Loss and the global sums
 * of phase 1 over the active features (V, Delta, VDeltaPrev, Tau, B,
 * VDelta into *globals); plx_swifttd_apply is the dense pass over all
 * features (phases 1 and 2, ResetGlobal). Same arguments and rules as
 * plx_swifttd_step; apply must follow reduce with the same active list. */
int plx_swifttd_reduce(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                       const uint32_t* active_idx, const float* active_val,
                       uint32_t n_active, const float* reward,
                       plx_td_globals* globals, float* v_out, void* scratch,
                       uint64_t scratch_bytes);
int plx_swifttd_apply(plx_ctx* ctx, uint64_t n_features, float* const* fields,
                      const uint32_t* active_idx, const float* active_val,
                      uint32_t n_active, plx_td_globals* globals, void* scratch,
                      uint64_t scratch_bytes);

#ifdef __cplusplus
}
#endif

#endif /* PLASTIX_B200_H */
