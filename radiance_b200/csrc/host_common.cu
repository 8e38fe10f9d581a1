// Host-side helpers shared by every entry point: error text, device queries, tensor maps.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

namespace rb_host {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cache[device] = n;
  }
  return cache[device];
}

static int g_sm_budget[64] = {0};

int sm_budget(int device) {
  const int n = num_sms(device);
  if (device < 0 || device >= 64 || g_sm_budget[device] <= 0 || g_sm_budget[device] >= n) return n;
  return g_sm_budget[device];
}

int set_sm_budget(int device, int sms) {
  if (device < 0 || device >= 64) return 0;
  const int prev = g_sm_budget[device];
  g_sm_budget[device] = sms < 0 ? 0 : sms;
  return prev;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// The tensor-map encoder is a driver call and needs a context current on this thread.  The runtime
// binds the device's primary context lazily, on a thread's first runtime call that needs one; a
// thread whose first call into this library encodes a tensor map (autograd's backward thread, for
// one) gets it bound here, with driver calls that are legal during stream capture.
static void bind_context() {
  static thread_local int bound = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || bound == dev) return;
  using GetCurrent = CUresult (*)(CUcontext*);
  using Retain = CUresult (*)(CUcontext*, CUdevice);
  using SetCurrent = CUresult (*)(CUcontext);
  static GetCurrent get_current = nullptr;
  static Retain retain = nullptr;
  static SetCurrent set_current = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && p)
      get_current = reinterpret_cast<GetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuDevicePrimaryCtxRetain", &p, cudaEnableDefault, &q) == cudaSuccess && p)
      retain = reinterpret_cast<Retain>(p);
    if (cudaGetDriverEntryPoint("cuCtxSetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess && p)
      set_current = reinterpret_cast<SetCurrent>(p);
  });
  if (get_current == nullptr || retain == nullptr || set_current == nullptr) return;
  CUcontext cur = nullptr;
  if (get_current(&cur) == CUDA_SUCCESS && cur == nullptr) {
    CUcontext primary = nullptr;  // the runtime's own context for this device (retained once per thread)
    if (retain(&primary, (CUdevice)dev) == CUDA_SUCCESS) set_current(primary);
  }
  bound = dev;
}

bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t cols, uint64_t rows,
                  uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  bind_context();
  auto enc = tensor_map_encoder();
  if (enc == nullptr) {
    set_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
    return false;
  }
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): base=%p cols=%llu rows=%llu ld=%llu box=%ux%u", (int)r, base,
              (unsigned long long)cols, (unsigned long long)rows, (unsigned long long)ld_bytes, box_cols, box_rows);
    return false;
  }
  return true;
}

}  // namespace rb_host

// Status words written by the kernels of each translation unit (read and cleared below).
extern "C" uint32_t rb_internal_quant_status(int clear);
extern "C" uint32_t rb_internal_gemm_status(int clear);

extern "C" {

const char* rb_nvfp4_last_error(void) { return rb_host::g_last_error; }

int rb_nvfp4_abi_version(void) { return RB_NVFP4_ABI_VERSION; }

int rb_nvfp4_set_sm_budget(int sms) { return rb_host::set_sm_budget(rb_host::current_device(), sms); }

int rb_nvfp4_device_status(int clear) {
  uint32_t s = rb_internal_quant_status(clear);
  uint32_t g = rb_internal_gemm_status(clear);
  return static_cast<int>(s != 0 ? s : g);
}

}  // extern "C"
