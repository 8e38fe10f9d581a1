// Shared device/host helpers for the NVFP4 kernels (sm_100a only).
//
// Every spin-wait in these kernels is bounded: a wait that runs past kWaitLimitCycles records an
// error code in the launch's status word and the kernel returns instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "radiance_b200 kernels are written for sm_100a (B200) only"
#endif

namespace rb {

// ~1 s at the B200's 1.965 GHz boost clock.
constexpr long long kWaitLimitCycles = 2000000000LL;

// Status codes written by kernels (host reads them through rb_nvfp4_device_status).
enum : uint32_t {
  kStatusOk = 0,
  kStatusTimeoutTma = 1,       // a TMA completion never arrived
  kStatusTimeoutMma = 2,       // an MMA commit never arrived
  kStatusTimeoutEpilogue = 3,  // the epilogue waited too long for the accumulator
  kStatusTimeoutProducer = 4,  // a producer waited too long for a free stage
  kStatusBadGroup = 5,         // a grouped-GEMM group descriptor broke the contract (group skipped)
  kStatusTmemBase = 6,         // a whole-TMEM allocation did not start at address 0 (GEMM skipped)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_status(uint32_t* status, uint32_t code) {
  if (status != nullptr) atomicCAS(status, 0u, code);
}

// ----------------------------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false after ~1 s (`limit`
// cycles; only the wait self-test passes a shorter limit).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > limit) return false;
  }
  return true;
}

// As mbar_wait, sleeping ~`ns` nanoseconds between polls: for long waits of warps that share a
// scheduler with a latency-critical warp (the GEMM's epilogue warps beside its MMA issuer).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns,
                                                long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > limit) return false;
    __nanosleep(ns);
  }
  return true;
}

// ----------------------------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ----------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                                 int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Plain (untiled) bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace rb

// ----------------------------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------------------------
namespace rb_host {

void set_error(const char* fmt, ...);
int num_sms(int device);
// The SMs this library's kernels size their grids for on `device`: all of them unless the caller
// set a smaller budget (rb_nvfp4_set_sm_budget), leaving the rest to concurrent kernels.
int sm_budget(int device);
int set_sm_budget(int device, int sms);
int current_device();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// 2-D row-major tensor map over `rows` x `cols` elements with `ld_bytes` between rows.
bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                  uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle);

}  // namespace rb_host
