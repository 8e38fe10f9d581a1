// The global scale (amax) for callers that cannot allocate device memory.
//
// rb_nvfp4_global_scale needs an 8-byte workspace from the caller.  Some callers have no way to
// provide one on the call path: code running where device allocation is not allowed (inside a
// host callback, where no CUDA call may allocate), plugin hosts whose execute step only receives
// buffers planned ahead of time, and plain C or FFI callers that hold device pointers but no
// device allocator.  This file gives them rb_nvfp4_global_scale_noalloc, which computes the same
// value using a fixed scratch array that lives in this library's device image instead of a
// caller-provided workspace.
//
// The scratch is a file-scope device array of kScratchWords 32-bit words (64 KiB plus 256 bytes;
// every GPU that loads the library holds it until the process exits): one ticket counter and one
// partial maximum per thread block.  Each block reduces a fixed chunk of kChunk elements, so one
// call can cover at most kMaxBlocks * kChunk = 2^31 elements; larger inputs are rejected.
//
// All calls on a device share the array and it keeps the last call's contents.  The ticket
// counter is cleared (one 4-byte memset on the caller's stream) at the start of every call; the
// partials need no clearing because every block writes its own slot before it takes a ticket.
// Two calls whose kernels overlap on the GPU (for example on two streams without ordering between
// them) race on the array and must not be issued.
#include <mutex>

#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

namespace rb_noalloc {

constexpr int kThreads = 512;
constexpr int64_t kChunk = 131072;  // elements per block (256 per thread)
constexpr int kMaxBlocks = 16384;
constexpr int kPartialBase = 64;    // word 0: ticket; words 64.. : per-block partial maxima
constexpr int kScratchWords = kPartialBase + kMaxBlocks;

static __device__ __align__(256) uint32_t g_scratch[kScratchWords];

// Max of |x| as fp32 bit patterns over one block's chunk (non-negative floats order like their
// bits, and NaN sorts above infinity, so the maximum propagates NaN as torch's amax does).
template <bool F32IN>
__device__ __forceinline__ uint32_t chunk_max(const void* x, int64_t rows, int64_t cols, int64_t ld, int64_t begin,
                                              int64_t end) {
  uint32_t m = 0;
  if (ld == cols && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (begin % 8) == 0) {
    constexpr int kPer = F32IN ? 4 : 8;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int64_t vb = begin / kPer, ve = end / kPer;
    for (int64_t i = vb + threadIdx.x; i < ve; i += kThreads) {
      const uint4 v = __ldg(xv + i);
      if constexpr (F32IN) {
        m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
      } else {
        const uint32_t h = __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                    __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu));
        m = max(m, max(h & 0xFFFFu, h >> 16) << 16);
      }
    }
    for (int64_t e = ve * kPer + threadIdx.x; e < end; e += kThreads) {
      if constexpr (F32IN) m = max(m, reinterpret_cast<const uint32_t*>(x)[e] & 0x7FFFFFFFu);
      else m = max(m, (uint32_t)(reinterpret_cast<const uint16_t*>(x)[e] & 0x7FFFu) << 16);
    }
  } else {
    for (int64_t e = begin + threadIdx.x; e < end; e += kThreads) {
      const int64_t r = e / cols, c = e - r * cols;
      if constexpr (F32IN) m = max(m, reinterpret_cast<const uint32_t*>(x)[r * ld + c] & 0x7FFFFFFFu);
      else m = max(m, (uint32_t)(reinterpret_cast<const uint16_t*>(x)[r * ld + c] & 0x7FFFu) << 16);
    }
  }
  return m;
}

__device__ __forceinline__ uint32_t block_max(uint32_t m, uint32_t* red) {
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < kThreads / 32 ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
  }
  return m;  // valid in warp 0
}

template <bool F32IN>
__global__ void __launch_bounds__(kThreads) global_scale_noalloc_kernel(const void* x, int64_t rows, int64_t cols,
                                                                          int64_t ld, uint32_t* scratch,
                                                                          float* gs_out) {
  __shared__ uint32_t red[kThreads / 32];
  __shared__ int is_last;
  const int64_t n = rows * cols;
  const int64_t begin = (int64_t)blockIdx.x * kChunk;
  const int64_t end = min(n, begin + kChunk);
  uint32_t m = block_max(chunk_max<F32IN>(x, rows, cols, ld, begin, end), red);
  if (threadIdx.x == 0) {
    scratch[kPartialBase + blockIdx.x] = m;
    __threadfence();
    is_last = atomicAdd(&scratch[0], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  m = 0;
  for (int i = threadIdx.x; i < (int)gridDim.x; i += kThreads) m = max(m, __ldcg(&scratch[kPartialBase + i]));
  __syncthreads();  // `red` is reused
  m = block_max(m, red);
  if (threadIdx.x == 0) {
    float gs = __fdiv_rn(__uint_as_float(m), 2688.0f);  // amax / (6 * 448), one IEEE divide
    gs = (gs < 1e-12f) ? 1e-12f : gs;
    *gs_out = gs;
    scratch[0] = 0u;
  }
}

// Device address of g_scratch, looked up once per device with that device current.
static uint32_t* scratch_ptr(int dev) {
  static uint32_t* ptrs[64] = {nullptr};
  static std::mutex mu;
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) {
      rb_host::set_error("nvfp4 global_scale_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<uint32_t*>(p);
  }
  return ptrs[dev];
}

}  // namespace rb_noalloc

extern "C" int rb_nvfp4_global_scale_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                             float* gs_out, void* stream) {
  using namespace rb_noalloc;
  if (gs_out == nullptr || (x == nullptr && rows * cols > 0)) {
    rb_host::set_error("nvfp4 global_scale_noalloc: null pointer argument");
    return RB_ERR_ARG;
  }
  if (dtype != RB_DTYPE_BF16 && dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 global_scale_noalloc: unsupported dtype %d", dtype);
    return RB_ERR_ARG;
  }
  if (rows <= 0 || cols <= 0 || ld < cols) {
    rb_host::set_error("nvfp4 global_scale_noalloc: bad shape rows=%lld cols=%lld ld=%lld", (long long)rows,
                       (long long)cols, (long long)ld);
    return RB_ERR_SHAPE;
  }
  const int64_t n = rows * cols;
  const int64_t blocks = (n + kChunk - 1) / kChunk;
  if (blocks > kMaxBlocks) {
    rb_host::set_error(
        "nvfp4 global_scale_noalloc: %lld elements exceed its limit of %lld (its fixed device scratch holds "
        "%d per-block partial maxima of %lld elements each); use rb_nvfp4_global_scale with a workspace",
        (long long)n, (long long)kMaxBlocks * kChunk, kMaxBlocks, (long long)kChunk);
    return RB_ERR_SHAPE;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) {
    rb_host::set_error("nvfp4 global_scale_noalloc: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  // The scratch used is the current device's, so x must live there too (a stream of another device
  // cannot be checked here; it must belong to the current device as well).
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, x) == cudaSuccess) {
    if ((attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) && attr.device != dev) {
      rb_host::set_error(
          "nvfp4 global_scale_noalloc: x is on device %d but the current device is %d; make x's device current "
          "(the call uses the current device's scratch)", attr.device, dev);
      return RB_ERR_ARG;
    }
  } else {
    cudaGetLastError();  // an unregistered host pointer is not an error for this check
  }
  uint32_t* scratch = scratch_ptr(dev);
  if (scratch == nullptr) return RB_ERR_CUDA;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(scratch, 0, sizeof(uint32_t), s);  // the ticket must start at zero
  if (e == cudaSuccess) {
    if (dtype == RB_DTYPE_BF16)
      global_scale_noalloc_kernel<false><<<(int)blocks, kThreads, 0, s>>>(x, rows, cols, ld, scratch, gs_out);
    else
      global_scale_noalloc_kernel<true><<<(int)blocks, kThreads, 0, s>>>(x, rows, cols, ld, scratch, gs_out);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 global_scale_noalloc launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}
