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

// RN(g / d) for d = 1 + exp(-g), two elements at a time, given nd = -d and s = RN(1/d).
// Markstein's correctly rounded division (P. Markstein, IBM J. R&D 34(1), 1990; Muller et al.,
// Handbook of Floating-Point Arithmetic, ch. 4): q = RN(g * s), then two residual corrections
// r = g - q*d, q += r*s, each one fused multiply-add on the packed f32x2 pipe; the first makes q
// faithful, the second, with a correctly rounded reciprocal, makes it the correctly rounded
// quotient.  That needs a finite g, a finite d and a normal residual, so the rare elements outside
// 2^-100 <= |g| < 2^100 and g > -64 (exp(64) < 2^93) -- signed zeros, subnormals, infinities, NaN,
// large negative gates whose d overflows -- take the IEEE divide.
__device__ __forceinline__ bool markstein_ok(float g) { return fabsf(g) >= 0x1p-100f && g > -64.0f && g < 0x1p100f; }

__device__ __forceinline__ float2 silu_quotient2(float2 g, float2 d, float2 nd, float2 s) {
  float2 q = __fmul2_rn(g, s);
  float2 r = __ffma2_rn(q, nd, g);
  q = __ffma2_rn(r, s, q);
  r = __ffma2_rn(q, nd, g);
  q = __ffma2_rn(r, s, q);
  if (!markstein_ok(g.x)) q.x = __fdiv_rn(g.x, d.x);
  if (!markstein_ok(g.y)) q.y = __fdiv_rn(g.y, d.y);
  return q;
}

// Two fp32 values -> two bf16 (round to nearest even), x in the low half.
__device__ __forceinline__ uint32_t bf16x2_bits(float2 v) {
  const __nv_bfloat162 b = __float22bfloat162_rn(v);
  return *reinterpret_cast<const uint32_t*>(&b);
}
__device__ __forceinline__ float2 bf16x2_float2(uint32_t w) { return make_float2(bf16_lo(w), bf16_hi(w)); }

// Two elements (the low and high bf16 of each word): (grad_g, grad_u) as bf16x2 words.  s = 1 / d is
// the correctly rounded reciprocal, the value the IEEE divide 1.0f / d gives.
__device__ __forceinline__ void swiglu_grad2(uint32_t dhw, uint32_t gw, uint32_t uw, uint32_t& ggw, uint32_t& guw) {
  const float2 dh = bf16x2_float2(dhw), g = bf16x2_float2(gw), u = bf16x2_float2(uw);
  const float2 d = make_float2(1.0f + expf(-g.x), 1.0f + expf(-g.y));
  const float2 s = make_float2(__frcp_rn(d.x), __frcp_rn(d.y));
  const float2 one = make_float2(1.0f, 1.0f);
  const float2 silu = bf16x2_float2(bf16x2_bits(silu_quotient2(g, d, make_float2(-d.x, -d.y), s)));  // F.silu(g)
  guw = bf16x2_bits(__fmul2_rn(dh, silu));                                      // grad_h * F.silu(g)
  const float2 t = bf16x2_float2(bf16x2_bits(__fmul2_rn(dh, u)));               // grad_h * u, bf16
  const float2 w = __ffma2_rn(g, __fadd2_rn(one, make_float2(-s.x, -s.y)), one);  // 1 + g * (1 - s)
  ggw = bf16x2_bits(__fmul2_rn(__fmul2_rn(t, s), w));                           // silu_backward(t, g)
}

// Thread layout: blockIdx.x and threadIdx.x pick an 8-unit chunk q of the hidden dimension (a chunk
// never straddles a 32-unit group), blockIdx.y a run of `rows_per_y` rows; a warp's 32 chunks of one
// row are contiguous in all three tensors.  No index division in the loop.
__global__ void __launch_bounds__(256, 6) swiglu_backward_kernel(const uint16_t* grad_h, int64_t ldgh, const uint16_t* gu,
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
        swiglu_grad2(dw[k], gw[k], uw[k], og[k], ou[k]);
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
  // One wave: as many 256-thread blocks as the SMs hold at once, each covering a run of rows for 256
  // chunks of the hidden dimension, so no SM idles through a partial last wave.
  static int resident[64] = {0};
  int& per_sm = resident[dev & 63];
  if (per_sm == 0 &&
      (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rb::swiglu_backward_kernel, 256, 0) != cudaSuccess ||
       per_sm < 1))
    per_sm = 1;
  const int64_t gx = (hidden / 8 + 255) / 256;
  int64_t gy = ((int64_t)per_sm * rb_host::sm_budget(dev)) / gx;
  if (gy < 1) gy = 1;
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
