// Global sum of an fp32 vector (reduction.cuh:8-44).
//
// The input is split into G equal chunks (G <= 8 x SM count, one resident
// wave); CTA b sums chunk b in fp64 (16-byte streaming loads, eight
// independent vectors in flight per thread), writes its partial to a scratch
// slot, and the CTA that finishes last adds the G partials in index order.
// The partition and the combine order depend only on n and the SM count, so
// the result is identical from run to run on a device model, unlike the fp32
// atomicAdd combine of the reference (reduction.cu:43); and the fp64
// accumulation keeps the relative error near 1e-12 even for 2^30 inputs,
// where an fp32 running sum loses ~1e-6.
#include <mutex>

#include "common.cuh"

namespace col {

// Library-owned stream-ordered memory pool of the current device.  Its
// release threshold keeps freed blocks mapped, so the per-call scratch
// allocation below is a cheap pool hit instead of a fresh mapping after
// every synchronisation (what the default pool, threshold 0, would do).
// Shared by every operator that needs stream-ordered scratch.
cudaError_t library_pool(cudaMemPool_t* pool) {
  constexpr int kMaxDevices = 64;
  static cudaMemPool_t pools[kMaxDevices] = {};
  static cudaError_t errors[kMaxDevices] = {};
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(flags[dev], [dev]() {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    cudaError_t err = cudaMemPoolCreate(&p, &props);
    if (err == cudaSuccess) {
      std::uint64_t keep = ~0ull;
      err = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pools[dev] = p;
    errors[dev] = err;
  });
  *pool = pools[dev];
  return errors[dev];
}

cudaError_t scratch_alloc(void** ptr, std::size_t bytes, cudaStream_t s) {
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(s, &capturing);
  if (e != cudaSuccess) return e;
  if (capturing != cudaStreamCaptureStatusNone) return cudaMallocAsync(ptr, bytes, s);
  cudaMemPool_t pool = nullptr;
  e = library_pool(&pool);
  if (e != cudaSuccess) return e;
  return cudaMallocFromPoolAsync(ptr, bytes, pool, s);
}

}  // namespace col

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 8;  // 16-byte loads in flight per thread
constexpr int kCtasPerSm = 8;                   // fallback: 256-thread CTAs per SM
constexpr std::uint64_t kChunkQuantum = 1024;   // elements: one float4 per thread
constexpr std::uint64_t kMinChunk = 4096;

struct Plan {
  std::uint64_t per_cta;
  unsigned ctas;
};

// STREAM: evict-first loads, for inputs larger than the L2 (a read-once
// stream should not push other data out); otherwise plain loads, which hit an
// input a previous kernel has just written (2^24 elements warm: 13.2 -> 8.7 us;
// cold inputs and inputs above the L2 read the same either way).
template <bool VEC, bool OUT_F64, bool STREAM = true>
__global__ void sum_kernel(const float* __restrict__ x, std::uint64_t n, std::uint64_t per_cta,
                           double* __restrict__ partials, unsigned* __restrict__ counter, void* out);

// CTAs of sum_kernel resident per SM on the current device (occupancy API,
// queried once per device); the one-wave grid is sm_count times this.
int resident_ctas_per_sm() {
  constexpr int kMaxDevices = 64;
  static int cached[kMaxDevices] = {};
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return kCtasPerSm;
  std::call_once(flags[dev], [dev]() {
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, sum_kernel<true, false>, kThreads,
                                                      0) != cudaSuccess ||
        blocks <= 0) {
      blocks = kCtasPerSm;
    }
    cached[dev] = blocks;
  });
  return cached[dev];
}

// One wave: at most sm_count x (CTAs resident per SM), every chunk the same
// size (a multiple of 1024 elements, so chunk starts keep 16-byte alignment),
// so all CTAs are resident at once and finish together.
Plan plan_for(std::uint64_t n) {
  const std::uint64_t target =
      static_cast<std::uint64_t>(col::device_info().sm_count) * resident_ctas_per_sm();
  std::uint64_t per = (n + target - 1) / target;
  per = (per + kChunkQuantum - 1) / kChunkQuantum * kChunkQuantum;
  if (per < kMinChunk) per = kMinChunk;
  Plan p;
  p.per_cta = per;
  p.ctas = static_cast<unsigned>((n + per - 1) / per);
  return p;
}

__device__ __forceinline__ double block_sum_f64(double v, double* sh) {
  v = col::warp_sum_f64(v);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x < 32) {
    s = (threadIdx.x < kThreads / 32) ? sh[threadIdx.x] : 0.0;
    s = col::warp_sum_f64(s);
  }
  __syncthreads();
  return s;  // valid in warp 0
}

// scratch layout: [0, ctas) doubles = partials, then one unsigned counter
// (zero on entry; the finishing CTA puts it back to zero).
template <bool VEC, bool OUT_F64, bool STREAM>
__global__ void __launch_bounds__(kThreads)
sum_kernel(const float* __restrict__ x, std::uint64_t n, std::uint64_t per_cta,
           double* __restrict__ partials, unsigned* __restrict__ counter, void* out) {
  __shared__ double sh[kThreads / 32];
  __shared__ bool is_last;
  col::grid_dependency_wait();
  const std::uint64_t begin = static_cast<std::uint64_t>(blockIdx.x) * per_cta;
  const std::uint64_t end = min(begin + per_cta, n);
  double acc = 0.0;
  if constexpr (VEC) {
    const float4* __restrict__ xv = reinterpret_cast<const float4*>(x + begin);
    const std::uint64_t nv = (end - begin) / 4;
    // Groups of kUnroll strided vectors, the last group predicated: every
    // group costs one memory round trip, including the ragged end.
    for (std::uint64_t i = threadIdx.x; i < nv; i += kUnroll * kThreads) {
      float4 q[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const std::uint64_t idx = i + static_cast<std::uint64_t>(j) * kThreads;
        if (idx < nv) {
          q[j] = STREAM ? col::ld_stream_f4(xv + idx) : col::ld_cached_f4(xv + idx);
        } else {
          q[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        acc += static_cast<double>(q[j].x);
        acc += static_cast<double>(q[j].y);
        acc += static_cast<double>(q[j].z);
        acc += static_cast<double>(q[j].w);
      }
    }
    for (std::uint64_t k = begin + nv * 4 + threadIdx.x; k < end; k += kThreads) {
      acc += static_cast<double>(x[k]);  // at most 3 trailing elements
    }
  } else {
    for (std::uint64_t k = begin + threadIdx.x; k < end; k += kThreads) {
      acc += static_cast<double>(STREAM ? __ldcs(x + k) : __ldg(x + k));
    }
  }
  const double cta_sum = block_sum_f64(acc, sh);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = cta_sum;
    __threadfence();
    const unsigned ticket = atomicAdd(counter, 1u);
    is_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // Fixed-order combine: thread t adds partials t, t+256, ... then the tree.
  double s = 0.0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += kThreads) {
    s += __ldcg(partials + b);
  }
  s = block_sum_f64(s, sh);
  if (threadIdx.x == 0) {
    if constexpr (OUT_F64) {
      *static_cast<double*>(out) = s;
    } else {
      *static_cast<float*>(out) = static_cast<float>(s);
    }
    *counter = 0u;
  }
}

template <bool OUT_F64>
int launch_sum(const float* x, void* out, std::uint64_t n, cudaStream_t s, double* partials,
               unsigned* counter) {
  const Plan p = plan_for(n);
  const bool stream = n * sizeof(float) > static_cast<std::uint64_t>(col::device_info().l2_bytes);
  const dim3 grid(p.ctas), block(kThreads);
  if (col::aligned16(x)) {
    return stream ? col::launch_serialised(sum_kernel<true, OUT_F64, true>, grid, block, 0, s, x, n,
                                           p.per_cta, partials, counter, out)
                  : col::launch_serialised(sum_kernel<true, OUT_F64, false>, grid, block, 0, s, x,
                                           n, p.per_cta, partials, counter, out);
  }
  return stream ? col::launch_serialised(sum_kernel<false, OUT_F64, true>, grid, block, 0, s, x, n,
                                         p.per_cta, partials, counter, out)
                : col::launch_serialised(sum_kernel<false, OUT_F64, false>, grid, block, 0, s, x, n,
                                         p.per_cta, partials, counter, out);
}

// Stream-ordered scratch: allocated and freed on the caller's stream, so
// concurrent calls on different streams never share it (col::scratch_alloc).
template <bool OUT_F64>
int reduce_with_pool_scratch(const float* x, void* out, std::uint64_t n, cudaStream_t s) {
  const Plan p = plan_for(n);
  const std::size_t bytes = static_cast<std::size_t>(p.ctas) * sizeof(double) + 16;
  void* scratch = nullptr;
  cudaError_t st = col::scratch_alloc(&scratch, bytes, s);
  if (st != cudaSuccess) return static_cast<int>(st);
  double* partials = static_cast<double*>(scratch);
  unsigned* counter = reinterpret_cast<unsigned*>(partials + p.ctas);
  st = cudaMemsetAsync(counter, 0, sizeof(unsigned), s);
  int rc = static_cast<int>(st);
  if (st == cudaSuccess) rc = launch_sum<OUT_F64>(x, out, n, s, partials, counter);
  const cudaError_t fst = cudaFreeAsync(scratch, s);
  if (rc == 0 && fst != cudaSuccess) rc = static_cast<int>(fst);
  return rc;
}

// Persistent scratch per (device, stream): sized once for the largest plan
// (one wave of CTAs), counter zeroed once when it is created and put back
// to zero by the finishing CTA of every launch.  Work on one stream is
// ordered, and different streams get different blocks, so the counter is
// zero whenever a launch starts and a call is a single kernel launch.  The
// block is created on the first call on a stream (cudaMalloc plus a memset
// on that stream); calls captured into a graph, more than kMaxStreamScratch
// streams, and cudaStreamPerThread (one handle naming a different stream on
// every host thread) use the stream-ordered pool path.
constexpr int kMaxStreamScratch = 256;

// Entries are keyed by the stream's process-unique id (cudaStreamGetId), not
// by its handle: a destroyed stream's handle value may be reused for a new
// stream, which must not inherit the old stream's block while work of the
// old one could still be pending.  A block is never freed; it lives until
// the process exits (at most kMaxStreamScratch of them).
struct StreamScratch {
  int device;
  unsigned long long stream_id;
  double* partials;
  unsigned* counter;
};

// Blocks for captured calls.  A captured call must not embed a stream's
// block (the graph may run on another stream, concurrently with that stream's
// own calls), so it takes a block of its own for good: kCaptureBlocks of them
// per device are made, counters zeroed and synchronised, by the first
// non-captured call on the device; once they are used up, captured calls take
// stream-ordered scratch (graph memory nodes and a counter memset).
constexpr int kCaptureBlocks = 64;

struct CaptureBlocks {
  double* base = nullptr;
  int next = 0;
  bool tried = false;
};

std::mutex capture_mu;
CaptureBlocks capture_blocks[64];

std::size_t block_stride(unsigned capacity) {
  return (static_cast<std::size_t>(capacity) * sizeof(double) + 256 + 255) / 256 * 256;
}

// Called outside any capture, with capture_mu held.
void make_capture_blocks(int dev, unsigned capacity, cudaStream_t s) {
  CaptureBlocks& cb = capture_blocks[dev & 63];
  if (cb.tried) return;
  cb.tried = true;
  const std::size_t stride = block_stride(capacity);
  void* base = nullptr;
  if (cudaMalloc(&base, stride * kCaptureBlocks) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  if (cudaMemsetAsync(base, 0, stride * kCaptureBlocks, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(base);
    return;
  }
  cb.base = static_cast<double*>(base);
}

bool capture_scratch(int dev, unsigned capacity, double** partials, unsigned** counter) {
  std::lock_guard<std::mutex> lock(capture_mu);
  CaptureBlocks& cb = capture_blocks[dev & 63];
  if (cb.base == nullptr || cb.next == kCaptureBlocks) return false;
  double* p = reinterpret_cast<double*>(reinterpret_cast<char*>(cb.base) +
                                        block_stride(capacity) * static_cast<std::size_t>(cb.next++));
  *partials = p;
  *counter = reinterpret_cast<unsigned*>(p + capacity);
  return true;
}

bool stream_scratch(cudaStream_t s, unsigned ctas, double** partials, unsigned** counter) {
  static std::mutex mu;
  static StreamScratch entries[kMaxStreamScratch];
  static int used = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const unsigned capacity = static_cast<unsigned>(col::device_info().sm_count) *
                            static_cast<unsigned>(resident_ctas_per_sm());
  if (ctas > capacity || s == cudaStreamPerThread) return false;
  // A captured call never uses the stream's block: the graph may later run on
  // another stream, concurrently with calls on this one, and the two would
  // share partials and counter.
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &capturing) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (capturing != cudaStreamCaptureStatusNone) {
    return capture_scratch(dev, capacity, partials, counter);
  }
  {
    std::lock_guard<std::mutex> lock(capture_mu);
    make_capture_blocks(dev, capacity, s);
  }
  unsigned long long id = 0;
  if (cudaStreamGetId(s, &id) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i) {
    if (entries[i].device == dev && entries[i].stream_id == id) {
      *partials = entries[i].partials;
      *counter = entries[i].counter;
      return true;
    }
  }
  if (used == kMaxStreamScratch) return false;
  void* block = nullptr;
  const std::size_t bytes = static_cast<std::size_t>(capacity) * sizeof(double) + 256;
  if (cudaMalloc(&block, bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  double* p = static_cast<double*>(block);
  unsigned* c = reinterpret_cast<unsigned*>(p + capacity);
  if (cudaMemsetAsync(c, 0, sizeof(unsigned), s) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(block);
    return false;
  }
  entries[used++] = StreamScratch{dev, id, p, c};
  *partials = p;
  *counter = c;
  return true;
}

template <bool OUT_F64>
int reduce_any(const float* x, void* out, std::uint64_t n, cudaStream_t s) {
  const Plan p = plan_for(n);
  double* partials = nullptr;
  unsigned* counter = nullptr;
  if (stream_scratch(s, p.ctas, &partials, &counter)) {
    return launch_sum<OUT_F64>(x, out, n, s, partials, counter);
  }
  return reduce_with_pool_scratch<OUT_F64>(x, out, n, s);
}

// reduction.cu:160-167 and :179-181: output NULL, or input NULL with n > 0,
// is cudaErrorInvalidValue; n == 0 writes 0.
int reduce_f32(const float* x, float* out, std::uint64_t n, void* stream) {
  if (out == nullptr || (x == nullptr && n != 0)) return static_cast<int>(cudaErrorInvalidValue);
  const cudaStream_t s = col::as_stream(stream);
  if (n == 0) return static_cast<int>(cudaMemsetAsync(out, 0, sizeof(float), s));
  return reduce_any<false>(x, out, n, s);
}

}  // namespace

COL_API int cuda_operator_reduction_v0(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}
COL_API int cuda_operator_reduction_v1(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}
COL_API int cuda_operator_reduction_v2(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}
COL_API int cuda_operator_reduction_v3(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}
COL_API int cuda_operator_reduction_v4(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}
COL_API int cuda_operator_reduction_v5(const float* input, float* output, uint64_t n, void* stream) {
  return reduce_f32(input, output, n, stream);
}

COL_API int cuda_operator_reduction_partial_f64(const float* input, double* partial, uint64_t n,
                                                void* stream) {
  if (partial == nullptr || (input == nullptr && n != 0)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  const cudaStream_t s = col::as_stream(stream);
  if (n == 0) return static_cast<int>(cudaMemsetAsync(partial, 0, sizeof(double), s));
  return reduce_any<true>(input, partial, n, s);
}

// ============================================================================
// Allocation-free variant of the global sum.
//
// Some callers cannot let a library allocate device memory: a serving process
// that reserved the whole device for its own allocator at start-up (any further
// allocation fails or fragments that arena), a host framework whose policy is
// that plugins never allocate, or a latency-critical loop where an allocator
// call may synchronise.  For them this entry point runs the same sum kernel
// with its scratch (one fp64 partial per CTA and a CTA counter) in a
// fixed-size array that lives in the library image itself: no cudaMalloc,
// cudaFree, pool or other allocating routine is ever called.
//
// Limits and rules, all stated to the caller in include/cuda_operator_lab.h:
//  * the array holds kNoAllocMaxCtas partials; each CTA sums a fixed chunk of
//    kNoAllocChunk elements, so n may not exceed kNoAllocMaxElements (2^28);
//    larger n is rejected with kErrNoAllocCapacity before anything is launched;
//  * every GPU that loads the library holds the array (128 KiB + 256 bytes)
//    until the process exits;
//  * all calls on a device share the one array: two calls whose work overlaps
//    on the GPU (different streams, no ordering between them) race and give
//    wrong sums; calls ordered on one stream are fine;
//  * the array keeps the previous call's contents, so each call clears the
//    counter (the only field that must start at zero) on its stream first;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture on the device.
// ============================================================================

namespace {

constexpr std::uint64_t kNoAllocChunk = 16384;  // elements per CTA
constexpr unsigned kNoAllocMaxCtas = 16384;
constexpr std::uint64_t kNoAllocMaxElements = kNoAllocChunk * kNoAllocMaxCtas;  // 2^28

// kNoAllocMaxCtas fp64 partials followed by the CTA counter (its own 256-byte
// line).  In host code this name is only a stand-in for the symbol: the
// kernel gets the device address found by noalloc_scratch_address().
static __device__ __align__(256) double g_noalloc_scratch[kNoAllocMaxCtas + 32];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device (the first call on that device); nullptr if the lookup failed.
cudaError_t noalloc_scratch_address(double** out) {
  constexpr int kMaxDevices = 64;
  static double* addrs[kMaxDevices] = {};
  static cudaError_t errors[kMaxDevices] = {};
  static std::once_flag flags[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(flags[dev], [dev]() {
    void* p = nullptr;
    errors[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    addrs[dev] = errors[dev] == cudaSuccess ? static_cast<double*>(p) : nullptr;
  });
  *out = addrs[dev];
  return errors[dev];
}

}  // namespace

COL_API int cuda_operator_lab_reduction_noalloc(const float* input, float* output, uint64_t n,
                                                void* stream) {
  if (output == nullptr || (input == nullptr && n != 0)) {
    return static_cast<int>(cudaErrorInvalidValue);
  }
  if (n > kNoAllocMaxElements) return col::kErrNoAllocCapacity;
  const cudaStream_t s = col::as_stream(stream);
  if (n == 0) return static_cast<int>(cudaMemsetAsync(output, 0, sizeof(float), s));
  double* scratch = nullptr;
  const cudaError_t e = noalloc_scratch_address(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  double* partials = scratch;
  unsigned* counter = reinterpret_cast<unsigned*>(scratch + kNoAllocMaxCtas);
  const cudaError_t ms = cudaMemsetAsync(counter, 0, sizeof(unsigned), s);
  if (ms != cudaSuccess) return static_cast<int>(ms);
  const unsigned ctas = static_cast<unsigned>((n + kNoAllocChunk - 1) / kNoAllocChunk);
  if (col::aligned16(input)) {
    sum_kernel<true, false><<<ctas, kThreads, 0, s>>>(input, n, kNoAllocChunk, partials, counter,
                                                      output);
  } else {
    sum_kernel<false, false><<<ctas, kThreads, 0, s>>>(input, n, kNoAllocChunk, partials, counter,
                                                       output);
  }
  return static_cast<int>(cudaGetLastError());
}
