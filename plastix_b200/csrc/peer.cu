// Peer memory for hand-offs between GPUs without a collective library call:
// buffers shared through CUDA IPC handles (one process per GPU), written by
// the producing kernel with plain stores over NVLink, and a bounded barrier
// kernel that tells every peer this GPU's stores are complete and waits for
// theirs.
#include <cstring>

#include "common.cuh"

namespace plx {
namespace {

__device__ __forceinline__ void st_release_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct PeerFlags {
  uint64_t* f[PLX_MAX_PEERS];  // f[p]: rank p's flag array (n entries)
};

// Thread p: publish epoch into rank p's flag slot for this rank, then wait
// (bounded) until rank p has published the same epoch into this rank's array.
__global__ void k_peer_barrier(PeerFlags fl, uint32_t n, uint32_t rank, uint64_t epoch,
                               uint64_t timeout_ns, int32_t* status) {
  const uint32_t p = threadIdx.x;
  if (p >= n) return;
  __threadfence_system();  // this GPU's earlier stores to peer memory first
  st_release_sys_u64(fl.f[p] + rank, epoch);
  const uint64_t* mine = fl.f[rank] + p;
  if (ld_acquire_sys_u64(mine) >= epoch) return;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t spin = 0;; ++spin) {
    if (ld_acquire_sys_u64(mine) >= epoch) return;
    if ((spin & 63u) == 63u && global_timer_ns() - t0 > timeout_ns) {
      record_status(status, kStatusTimeout);
      return;
    }
  }
}

}  // namespace
}  // namespace plx

using namespace plx;

static_assert(sizeof(cudaIpcMemHandle_t) <= PLX_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" int plx_peer_alloc(plx_ctx* ctx, size_t bytes, void** ptr, void* ipc_handle) {
  PLX_CHECK_ARG(ctx && ptr && ipc_handle && bytes, "ctx, ptr, ipc_handle and bytes required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  void* p = nullptr;
  PLX_TRY_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return check_cuda(e, "plx_peer_alloc");
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return PLX_OK;
}

extern "C" int plx_peer_free(plx_ctx* ctx, void* ptr) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (ptr) PLX_TRY_CUDA(cudaFree(ptr));
  return PLX_OK;
}

extern "C" int plx_peer_open(plx_ctx* ctx, const void* ipc_handle, void** ptr) {
  PLX_CHECK_ARG(ctx && ipc_handle && ptr, "ctx, ipc_handle and ptr required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  PLX_TRY_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return PLX_OK;
}

extern "C" int plx_peer_close(plx_ctx* ctx, void* ptr) {
  PLX_CHECK_ARG(ctx, "ctx is required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (ptr) PLX_TRY_CUDA(cudaIpcCloseMemHandle(ptr));
  return PLX_OK;
}

extern "C" int plx_peer_barrier(plx_ctx* ctx, uint64_t* const* flags, uint32_t n,
                                uint32_t rank, uint64_t epoch) {
  PLX_CHECK_ARG(ctx && flags, "ctx and flags are required");
  PLX_CHECK_ARG(n >= 1 && n <= PLX_MAX_PEERS && rank < n, "bad rank %u of %u", rank, n);
  PeerFlags fl{};
  for (uint32_t p = 0; p < n; ++p) {
    PLX_CHECK_ARG(flags[p], "flags[%u] is NULL", p);
    fl.f[p] = flags[p];
  }
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  k_peer_barrier<<<1, 32, 0, ctx->stream>>>(fl, n, rank, epoch, ctx->timeout_ns, ctx->d_status);
  PLX_LAUNCH_CHECK("k_peer_barrier");
  return PLX_OK;
}

extern "C" int plx_copy_device(plx_ctx* ctx, void* dst, const void* src, size_t bytes) {
  PLX_CHECK_ARG(ctx && (bytes == 0 || (dst && src)), "ctx, dst and src are required");
  PLX_TRY_CUDA(cudaSetDevice(ctx->device));
  if (bytes) PLX_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream));
  return PLX_OK;
}
