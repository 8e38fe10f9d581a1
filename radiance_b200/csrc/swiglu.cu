// SwiGLU backward in one pass, with the global scale of its output.
//
// radiance's FFN computes h = F.silu(g) * u (src/radiance/model/ffn.py:32); autograd's backward of
// that line is grad_u = grad_h * F.silu(g) and grad_g = silu_backward(grad_h * u, g), each torch op a
// full pass over (tokens x hidden) bf16 tensors, and the gate/up linear then reads grad_gu once more
// for its global scale.  This kernel reads grad_h and the saved pre-activations once, writes grad_gu
// in the interleaved [32 gate | 32 up] column order of the gate/up operand, and reduces
// max |grad_gu| into the global scale (quantize.py:205-213) on the way.
//
// Every value is computed with the roundings of the eager torch ops it replaces: bf16 inputs
// widened to fp32, silu(g) = g / (1 + exp(-g)) rounded to bf16, products rounded to bf16, and
// silu_backward's dy * s * (1 + g * (1 - s)) with s = 1 / (1 + exp(-g)), evaluated in fp32 and rounded
// to bf16 once.  tests/test_swiglu_gpu.py checks the result against those torch ops bit for bit.
#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

namespace rb {

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf16_bits(float f) {
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// One element: (grad_g, grad_u) as bf16 bit patterns.
__device__ __forceinline__ void swiglu_grad(float dh, float g, float u, uint32_t& gg, uint32_t& gu) {
  const float e = expf(-g);
  const float d = 1.0f + e;
  const float silu = __uint_as_float(bf16_bits(__fdiv_rn(g, d)) << 16);  // F.silu(g), bf16
  gu = bf16_bits(dh * silu);                                             // grad_h * F.silu(g)
  const float t = __uint_as_float(bf16_bits(dh * u) << 16);              // grad_h * u, bf16
  const float s = __fdiv_rn(1.0f, d);
  gg = bf16_bits(t * s * __fmaf_rn(g, 1.0f - s, 1.0f));                  // silu_backward(t, g)
}

// Thread layout: blockIdx.x and threadIdx.x pick an 8-unit chunk q of the hidden dimension (a chunk
// never straddles a 32-unit group), blockIdx.y a run of `rows_per_y` rows; a warp's 32 chunks of one
// row are contiguous in all three tensors.  No index division in the loop.
__global__ void __launch_bounds__(256) swiglu_backward_kernel(const uint16_t* grad_h, int64_t ldgh, const uint16_t* gu,
                                                              int64_t ldgu, int64_t rows, int64_t hidden,
                                                              int64_t rows_per_y, uint16_t* grad_gu, int64_t ldgg,
                                                              uint32_t* ws, float* gs_out) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_y;
  const int64_t r1 = min(rows, r0 + rows_per_y);
  uint32_t m = 0;  // max of |grad_gu| bf16 bit patterns, two halves packed
  if (q < hidden / 8) {
    const int64_t c = (8 * q) >> 5, j0 = (8 * q) & 31;
    const uint16_t* ph = grad_h + r0 * ldgh + 8 * q;
    const uint16_t* pg = gu + r0 * ldgu + 64 * c + j0;
    uint16_t* po = grad_gu + r0 * ldgg + 64 * c + j0;
    for (int64_t r = r0; r < r1; ++r, ph += ldgh, pg += ldgu, po += ldgg) {
      const uint4 dh = __ldg(reinterpret_cast<const uint4*>(ph));
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(pg));
      const uint4 uv = __ldg(reinterpret_cast<const uint4*>(pg + 32));
      const uint32_t dw[4] = {dh.x, dh.y, dh.z, dh.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
      const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
      uint32_t og[4], ou[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t g0, u0, g1, u1;
        swiglu_grad(bf16_lo(dw[k]), bf16_lo(gw[k]), bf16_lo(uw[k]), g0, u0);
        swiglu_grad(bf16_hi(dw[k]), bf16_hi(gw[k]), bf16_hi(uw[k]), g1, u1);
        og[k] = g0 | (g1 << 16);
        ou[k] = u0 | (u1 << 16);
        m = __vmaxu2(m, __vmaxu2(og[k] & 0x7FFF7FFFu, ou[k] & 0x7FFF7FFFu));
      }
      *reinterpret_cast<uint4*>(po) = make_uint4(og[0], og[1], og[2], og[3]);
      *reinterpret_cast<uint4*>(po + 32) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    }
  }
  // max |x| bits -> fp32 bits, block maximum, one atomic per block; the last block converts.
  m = max(m & 0xFFFFu, m >> 16) << 16;
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t red[8];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = max(m, red[w]);
    atomicMax(&ws[0], m);
    __threadfence();
    last = atomicAdd(&ws[1], 1u) == gridDim.x * gridDim.y - 1;
    if (last) {
      __threadfence();
      const uint32_t mb = atomicExch(&ws[0], 0u);
      atomicExch(&ws[1], 0u);
      float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);  // amax / (6 * 448), one IEEE divide
      *gs_out = (gs < 1e-12f) ? 1e-12f : gs;
    }
  }
}

}  // namespace rb

extern "C" int rb_nvfp4_swiglu_backward(const void* grad_h, int64_t ldgh, const void* gu, int64_t ldgu, int64_t rows,
                                        int64_t hidden, void* grad_gu, int64_t ldgg, float* gs_out, void* workspace,
                                        void* stream) {
  if (grad_h == nullptr || gu == nullptr || grad_gu == nullptr || gs_out == nullptr || workspace == nullptr) {
    rb_host::set_error("nvfp4 swiglu_backward: null pointer argument");
    return RB_ERR_ARG;
  }
  if (rows <= 0 || hidden <= 0 || hidden % 32 != 0 || ldgh < hidden || ldgu < 2 * hidden || ldgg < 2 * hidden) {
    rb_host::set_error("nvfp4 swiglu_backward needs hidden %% 32 == 0 and row strides ldgh >= hidden, "
                       "ldgu, ldgg >= 2 * hidden, got rows=%lld hidden=%lld", (long long)rows, (long long)hidden);
    return RB_ERR_SHAPE;
  }
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(grad_h) || misaligned(gu) || misaligned(grad_gu) || (ldgh % 8) || (ldgu % 8) || (ldgg % 8) ||
      (reinterpret_cast<uintptr_t>(workspace) & 7)) {
    rb_host::set_error("nvfp4 swiglu_backward: tensors must be 16-byte aligned with row strides a multiple of 8 "
                       "elements, the workspace 8-byte aligned");
    return RB_ERR_ARG;
  }
  const int dev = rb_host::current_device();
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) {
    rb_host::set_error("nvfp4 swiglu_backward: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  // About eight 256-thread blocks per SM, each covering a run of rows for 256 chunks of the hidden
  // dimension.
  const int64_t gx = (hidden / 8 + 255) / 256;
  int64_t gy = (8 * (int64_t)rb_host::sm_budget(dev) + gx - 1) / gx;
  if (gy > rows) gy = rows;
  if (gy > 65535) gy = 65535;
  const int64_t rows_per_y = (rows + gy - 1) / gy;
  gy = (rows + rows_per_y - 1) / rows_per_y;
  rb::swiglu_backward_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint16_t*>(grad_h), ldgh, reinterpret_cast<const uint16_t*>(gu), ldgu, rows, hidden,
      rows_per_y, reinterpret_cast<uint16_t*>(grad_gu), ldgg, reinterpret_cast<uint32_t*>(workspace), gs_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 swiglu_backward launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}
