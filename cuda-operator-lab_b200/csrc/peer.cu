// Peer memory of the gathering GEMM (cuda_operator_gemm_swiglu_allgather_bf16):
// buffers shared between the processes of one node (one process per GPU)
// through CUDA IPC, and a flag barrier over NVLink that tells every rank when
// the other ranks' stores into its buffer are complete.
//
// Barrier protocol.  Each rank owns an array of `world` 32-bit flags in its
// shared buffer; slot j holds the epoch of the last barrier rank j arrived at.
// Arriving at epoch e, rank r writes e into slot r of every rank's array
// (release, system scope) and then waits until every slot of its own array
// holds e or later (acquire, system scope).  Stream order puts the barrier
// after the GEMM whose peer stores it publishes, and the GEMM's epilogue
// threads fence at system scope before they exit.  Epochs only grow, so no
// flag is ever reset.  The wait is bounded: on timeout the kernel sets a bit
// of the peer status word (cuda_operator_lab_peer_status) and returns.

#include <cstring>

#include "common.cuh"

namespace {

__device__ unsigned g_peer_status;

constexpr unsigned kStatusBarrierTimeout = 1u;
constexpr int kMaxRanks = 8;

struct FlagArrays {
  unsigned* flags[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One warp; thread t announces this rank to rank t and waits for rank t.
__global__ void __launch_bounds__(32)
peer_barrier_kernel(FlagArrays f, int rank, int world, unsigned epoch,
                    unsigned long long timeout_ns) {
  const int t = static_cast<int>(threadIdx.x);
  if (t >= world) return;
  __threadfence_system();
  st_release_sys(f.flags[t] + rank, epoch);
  const unsigned* mine = f.flags[rank] + t;
  const unsigned long long start = globaltimer_ns();
  while (static_cast<int>(ld_acquire_sys(mine) - epoch) < 0) {
    if (globaltimer_ns() - start > timeout_ns) {
      atomicOr(&g_peer_status, kStatusBarrierTimeout);
      return;
    }
    __nanosleep(100);
  }
}

}  // namespace

// Size of the opaque handle cuda_operator_lab_peer_alloc writes.
COL_API uint64_t cuda_operator_lab_peer_handle_bytes(void) {
  return sizeof(cudaIpcMemHandle_t);
}

// A zero-filled device allocation of `bytes` on the current device that other
// processes can map: *ptr receives the local address, `handle`
// (cuda_operator_lab_peer_handle_bytes() bytes) the handle to send to them.
COL_API int cuda_operator_lab_peer_alloc(uint64_t bytes, void** ptr, void* handle) {
  if (bytes == 0 || ptr == nullptr || handle == nullptr) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
  }
  return static_cast<int>(e);
}

// Maps another process's allocation (its handle) into this process; the
// address is valid in kernels of the current device (peer access over NVLink).
COL_API int cuda_operator_lab_peer_open(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

COL_API int cuda_operator_lab_peer_close(void* ptr) {
  if (ptr == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(cudaIpcCloseMemHandle(ptr));
}

COL_API int cuda_operator_lab_peer_free(void* ptr) {
  if (ptr == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  return static_cast<int>(cudaFree(ptr));
}

// Barrier of `world` ranks at `epoch` on `stream`: flag_arrays[j] is rank j's
// flag array (uint32[world], 4-byte aligned) as mapped in this process.  Later
// work on the stream sees every store the other ranks made before their
// barrier launch.  A wait longer than timeout_ns sets bit 1 of the peer status
// word instead of hanging.
COL_API int cuda_operator_lab_peer_barrier(void* const* flag_arrays, int rank, int world,
                                           uint32_t epoch, uint64_t timeout_ns, void* stream) {
  if (flag_arrays == nullptr || world < 1 || world > kMaxRanks || rank < 0 || rank >= world) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  FlagArrays f;
  std::memset(&f, 0, sizeof(f));
  for (int j = 0; j < world; ++j) {
    if (flag_arrays[j] == nullptr || (reinterpret_cast<std::uintptr_t>(flag_arrays[j]) & 3u)) {
      return static_cast<int>(cudaErrorInvalidValue);
    }
    f.flags[j] = static_cast<unsigned*>(flag_arrays[j]);
  }
  peer_barrier_kernel<<<1, 32, 0, col::as_stream(stream)>>>(f, rank, world, epoch, timeout_ns);
  return static_cast<int>(cudaGetLastError());
}

// Reads (and with `clear`, zeroes) the peer status word of the current device
// after synchronising it: bit 1 = a barrier wait timed out.
COL_API int cuda_operator_lab_peer_status(unsigned int* status, int clear) {
  if (status == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemcpyFromSymbol(status, g_peer_status, sizeof(unsigned));
  if (e != cudaSuccess) return static_cast<int>(e);
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_peer_status, &zero, sizeof(unsigned));
  }
  return static_cast<int>(e);
}
