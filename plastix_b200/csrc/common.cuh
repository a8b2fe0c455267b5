// Shared device helpers for the sm_100a kernels: error plumbing, the
// mbarrier / bulk-copy (TMA, non-tensor) primitives used by the streaming
// sweeps, and bounded waits that record a status instead of hanging.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/plastix_b200.h"

namespace plx {

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local message, int status codes).
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

#define PLX_TRY_CUDA(expr)                                                     \
  do {                                                                         \
    cudaError_t plx_e_ = (expr);                                               \
    if (plx_e_ != cudaSuccess) return ::plx::check_cuda(plx_e_, #expr);        \
  } while (0)

#define PLX_CHECK_ARG(cond, ...)                                               \
  do {                                                                         \
    if (!(cond)) return ::plx::set_error(PLX_ERR_ARG, __VA_ARGS__);            \
  } while (0)

#define PLX_LAUNCH_CHECK(what)                                                 \
  do {                                                                         \
    cudaError_t plx_e_ = cudaGetLastError();                                   \
    if (plx_e_ != cudaSuccess) return ::plx::check_cuda(plx_e_, what);         \
  } while (0)

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Device status word values (written by kernels whose waits time out).
enum DeviceStatus : int32_t {
  kStatusOk = 0,
  kStatusTimeout = 1,   // a bounded wait expired
  kStatusBadIndex = 2,  // a connection named a unit outside the given array
  kStatusBadPlan = 3,   // a sweep was given an invalid plan
};

// ---------------------------------------------------------------------------
// Device primitives
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the given phase parity, giving up after `timeout_ns` of wall
// time. Returns false on timeout (the caller records the status and skips the
// work that depended on the data).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity,
                                                  uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 63u && global_timer_ns() - t0 > timeout_ns)
      return false;
  }
}

// Bulk (non-tensor) asynchronous copy global -> shared, completion signalled
// on `bar` through the transaction count. dst, src and bytes must be 16-byte
// multiples / aligned.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src_gmem,
                                          uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Bulk asynchronous copy shared -> global (bulk-group completion).
__device__ __forceinline__ void bulk_store(void* dst_gmem, const void* src_smem,
                                           uint32_t bytes) {
  asm volatile(
      "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
          dst_gmem),
      "r"(smem_addr(src_smem)), "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// L2 cache policies for per-instruction hints: streamed connection data is
// marked evict-first, the gathered activation array evict-last, so the
// streams do not push the small, much re-read activation array out of L2.
// The hints change no state beyond the accesses that carry them.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void* p, uint64_t pol) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ float ld_keep_f32(const float* p, uint64_t pol) {
  float v;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
      : "=f"(v)
      : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void st_stream_v4(void* p, float4 v, uint64_t pol) {
  asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;"
               ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "l"(pol)
               : "memory");
}

// Asks the TMA unit to bring [p, p + bytes) into L2 (no completion, no data
// returned). p and bytes must be multiples of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes)
               : "memory");
}
// The same with an L2 cache policy for the prefetched lines.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p),
               "r"(bytes), "l"(pol)
               : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before subsequent
// async-proxy (bulk store) reads of the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void record_status(int32_t* status, int32_t code) {
  if (status) atomicCAS(status, kStatusOk, code);
}

// ---------------------------------------------------------------------------
// Apply rules of the row sweeps (one value per destination / source row).
// Reference evaluation order, separate roundings.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr bool apply_reads_value(int kind) {
  return kind == PLX_APPLY_IPC_ERROR || kind == PLX_APPLY_SIGMOID_GRAD ||
         kind == PLX_APPLY_TANH_GRAD;
}

template <int APPLY>
__device__ __forceinline__ float apply_value(float acc, float v) {
  if constexpr (APPLY == PLX_APPLY_IDENTITY) {
    return acc;  // traits.hpp:115-117
  } else if constexpr (APPLY == PLX_APPLY_SIGMOID) {
    // mlp_xor.cpp:24-26. exp in double precision, rounded once to float: the
    // correctly rounded single-precision exponential (up to rare near-halfway
    // cases), which is also what the host's expf returns to within its
    // half-ulp accuracy, so long training runs do not drift from the reference.
    return 1.0f / __fadd_rn(1.0f, (float)exp(-(double)acc));
  } else if constexpr (APPLY == PLX_APPLY_TANH) {
    return tanhf(acc);
  } else if constexpr (APPLY == PLX_APPLY_SIGMOID_GRAD) {
    return __fmul_rn(__fmul_rn(acc, v), __fsub_rn(1.0f, v));  // mlp_xor.cpp:43-46
  } else if constexpr (APPLY == PLX_APPLY_TANH_GRAD) {
    const float t = tanhf(v);  // ipc_multilayer.cpp:128-131,170-175
    return __fmul_rn(__fsub_rn(1.0f, __fmul_rn(t, t)), acc);
  } else {
    return __fsub_rn(v, acc);  // PLX_APPLY_IPC_ERROR, ipc_multilayer.cpp:147-150
  }
}

template <typename T>
__device__ __forceinline__ T ldg_nc(const T* p) {
  return __ldg(p);
}

}  // namespace plx

// Opaque context: one device, one stream, a device status word.
struct plx_ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  int num_sms = 0;
  int32_t* d_status = nullptr;  // device word written by bounded waits
  uint32_t* d_queue = nullptr;  // work counter of the warp sweeps (same allocation)
  uint64_t timeout_ns = 2000000000ull;
  uint32_t* d_counters = nullptr;  // per-window counters of the sliced hand-off
  size_t counters_cap = 0;
};

// The context's counter array, grown (never shrunk) to at least n words.
int ctx_counters(plx_ctx* ctx, size_t n, uint32_t** out);
