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

// One element pair of the forward: h = bf16(bf16(silu(g)) * u) as a bf16x2 word.  The product of
// two bf16 values is exact in fp32, so one bf16 multiply rounds it as torch's fp32 product rounded
// to bf16 does.
__device__ __forceinline__ uint32_t swiglu_h2(uint32_t gw, uint32_t uw) {
  const float2 g = bf16x2_float2(gw);
  const float2 d = make_float2(1.0f + expf(-g.x), 1.0f + expf(-g.y));
  const float2 s = make_float2(__frcp_rn(d.x), __frcp_rn(d.y));
  const uint32_t silu = bf16x2_bits(silu_quotient2(g, d, make_float2(-d.x, -d.y), s));  // F.silu(g)
  const __nv_bfloat162 h = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&silu),
                                      *reinterpret_cast<const __nv_bfloat162*>(&uw));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Where a SwiGLU pair lives: the gate value of (row r, hidden unit j) at
// gate[r * ld + (j / 32) * blk + j % 32] and the up value at the same offset from gate + du.
//   interleaved, the gate/up GEMM's [32 gate | 32 up] column order:  du = 32,      blk = 64;
//   split, radiance's [gate | up] halves (BatchedExperts, ffn.py:148-153): du = hidden, blk = 32.
// The backward writes grad_gate / grad_up with the same scheme (dug, blko, ldo).
struct SwigluArgs {
  const uint16_t* gate;
  int64_t du, ld, blk;        // pre-activations
  const uint16_t* grad_h;     // backward: upstream gradient, rows x hidden, row stride ldh
  uint16_t* h;                // forward: the activation, rows x hidden, row stride ldh
  int64_t ldh;
  uint16_t* grad_gate;        // backward outputs
  int64_t dug, ldo, blko;
  int64_t rows, hidden, rows_per_y;
  uint32_t* ws;               // {max bits, finished blocks}: zero on entry, left zero
  float* gs_out;              // global scale of h (forward) or of the gradient (backward)
};

// Thread layout: blockIdx.x and threadIdx.x pick an 8-unit chunk q of the hidden dimension (a chunk
// never straddles a 32-unit group), blockIdx.y a run of `rows_per_y` rows; a warp's 32 chunks of one
// row are contiguous in every tensor of the interleaved and split layouts.  No index division in
// the loop.
// kBlk: the group stride of both layouts when it is a compile-time constant (64: the interleaved
// layout, whose up offset is then 32), or 0 to read blk, du and the output scheme from `a`.
template <bool kBwd, int kBlk>
__global__ void __launch_bounds__(256, 6) swiglu_kernel(const SwigluArgs a) {
  const int64_t blk = kBlk ? kBlk : a.blk, du = kBlk ? 32 : a.du;
  const int64_t blko = kBlk ? kBlk : a.blko, dug = kBlk ? 32 : a.dug;
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r0 = (int64_t)blockIdx.y * a.rows_per_y;
  const int64_t r1 = min(a.rows, r0 + a.rows_per_y);
  uint32_t m = 0;  // max of |output| bf16 bit patterns, two halves packed
  if (q < a.hidden / 8) {
    const int64_t c = (8 * q) >> 5, j0 = (8 * q) & 31;
    const uint16_t* pg = a.gate + r0 * a.ld + c * blk + j0;
    if constexpr (kBwd) {
      const uint16_t* ph = a.grad_h + r0 * a.ldh + 8 * q;
      uint16_t* po = a.grad_gate + r0 * a.ldo + c * blko + j0;
      for (int64_t r = r0; r < r1; ++r, ph += a.ldh, pg += a.ld, po += a.ldo) {
        const uint4 dh = __ldg(reinterpret_cast<const uint4*>(ph));
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(pg));
        const uint4 uv = __ldg(reinterpret_cast<const uint4*>(pg + du));
        const uint32_t dw[4] = {dh.x, dh.y, dh.z, dh.w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
        const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t og[4], ou[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          swiglu_grad2(dw[k], gw[k], uw[k], og[k], ou[k]);
          m = __vmaxu2(m, __vmaxu2(og[k] & 0x7FFF7FFFu, ou[k] & 0x7FFF7FFFu));
        }
        *reinterpret_cast<uint4*>(po) = make_uint4(og[0], og[1], og[2], og[3]);
        *reinterpret_cast<uint4*>(po + dug) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
      }
    } else {
      uint16_t* ph = a.h + r0 * a.ldh + 8 * q;
      for (int64_t r = r0; r < r1; ++r, ph += a.ldh, pg += a.ld) {
        const uint4 gv = __ldg(reinterpret_cast<const uint4*>(pg));
        const uint4 uv = __ldg(reinterpret_cast<const uint4*>(pg + du));
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
        uint32_t hw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          hw[k] = swiglu_h2(gw[k], uw[k]);
          m = __vmaxu2(m, hw[k] & 0x7FFF7FFFu);
        }
        *reinterpret_cast<uint4*>(ph) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      }
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
    atomicMax(&a.ws[0], m);
    __threadfence();
    last = atomicAdd(&a.ws[1], 1u) == gridDim.x * gridDim.y - 1;
    if (last) {
      __threadfence();
      const uint32_t mb = atomicExch(&a.ws[0], 0u);
      atomicExch(&a.ws[1], 0u);
      float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);  // amax / (6 * 448), one IEEE divide
      *a.gs_out = (gs < 1e-12f) ? 1e-12f : gs;
    }
  }
}

}  // namespace rb

namespace {

bool swiglu_misaligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

// Checks shared by the entry points, then one wave of 256-thread blocks: as many as the SMs hold at
// once, each covering a run of rows for 256 chunks of the hidden dimension, so no SM idles through a
// partial last wave.
template <bool kBwd>
int swiglu_launch(rb::SwigluArgs& a, const char* what, void* workspace, void* stream) {
  if (a.gate == nullptr || a.gs_out == nullptr || workspace == nullptr ||
      (kBwd ? (a.grad_h == nullptr || a.grad_gate == nullptr) : a.h == nullptr)) {
    rb_host::set_error("%s: null pointer argument", what);
    return RB_ERR_ARG;
  }
  const int64_t groups = a.hidden / 32;
  // The row extent a layout reaches: groups of 32 units `blk` apart, plus the up offset.
  const auto extent = [&](int64_t du, int64_t blk) { return (groups - 1) * blk + 32 + du; };
  if (a.rows <= 0 || a.hidden <= 0 || a.hidden % 32 != 0 || a.blk < 32 || a.du < 0 || a.ldh < a.hidden ||
      a.ld < extent(a.du, a.blk) || (kBwd && (a.blko < 32 || a.dug < 0 || a.ldo < extent(a.dug, a.blko)))) {
    rb_host::set_error("%s needs hidden %% 32 == 0, group strides >= 32 and row strides that hold every group, got "
                       "rows=%lld hidden=%lld", what, (long long)a.rows, (long long)a.hidden);
    return RB_ERR_SHAPE;
  }
  if (swiglu_misaligned(a.gate) || (a.ld % 8) || (a.blk % 8) || (a.du % 8) || (a.ldh % 8) ||
      swiglu_misaligned(kBwd ? static_cast<const void*>(a.grad_h) : static_cast<const void*>(a.h)) ||
      (kBwd && (swiglu_misaligned(a.grad_gate) || (a.ldo % 8) || (a.blko % 8) || (a.dug % 8))) ||
      (reinterpret_cast<uintptr_t>(workspace) & 7)) {
    rb_host::set_error("%s: tensors must be 16-byte aligned with strides and offsets a multiple of 8 elements, the "
                       "workspace 8-byte aligned", what);
    return RB_ERR_ARG;
  }
  const int dev = rb_host::current_device();
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) {
    rb_host::set_error("%s: the current device is not an sm_100 GPU", what);
    return RB_ERR_DEVICE;
  }
  // The interleaved layout (in and out) runs the instantiation with its strides as constants.
  const bool interleaved = a.blk == 64 && a.du == 32 && (!kBwd || (a.blko == 64 && a.dug == 32));
  const auto kernel = interleaved ? rb::swiglu_kernel<kBwd, 64> : rb::swiglu_kernel<kBwd, 0>;
  static int resident[2][2][64] = {{{0}}};
  int& per_sm = resident[kBwd ? 1 : 0][interleaved ? 1 : 0][dev & 63];
  if (per_sm == 0 &&
      (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess || per_sm < 1))
    per_sm = 1;
  const int64_t gx = (a.hidden / 8 + 255) / 256;
  int64_t gy = ((int64_t)per_sm * rb_host::sm_budget(dev)) / gx;
  if (gy < 1) gy = 1;
  if (gy > a.rows) gy = a.rows;
  if (gy > 65535) gy = 65535;
  a.rows_per_y = (a.rows + gy - 1) / gy;
  gy = (a.rows + a.rows_per_y - 1) / a.rows_per_y;
  a.ws = reinterpret_cast<uint32_t*>(workspace);
  kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // namespace

extern "C" int rb_nvfp4_swiglu_backward(const void* grad_h, int64_t ldgh, const void* gu, int64_t ldgu, int64_t rows,
                                        int64_t hidden, void* grad_gu, int64_t ldgg, float* gs_out, void* workspace,
                                        void* stream) {
  rb::SwigluArgs a = {};
  a.gate = reinterpret_cast<const uint16_t*>(gu);
  a.du = 32;
  a.ld = ldgu;
  a.blk = 64;
  a.grad_h = reinterpret_cast<const uint16_t*>(grad_h);
  a.ldh = ldgh;
  a.grad_gate = reinterpret_cast<uint16_t*>(grad_gu);
  a.dug = 32;
  a.ldo = ldgg;
  a.blko = 64;
  a.rows = rows;
  a.hidden = hidden;
  a.gs_out = gs_out;
  return swiglu_launch<true>(a, "nvfp4 swiglu_backward", workspace, stream);
}

// Element offset of `p` from `base` (bf16 elements), or -1 when p lies below base.
static int64_t elem_offset(const void* base, const void* p) {
  const intptr_t d = reinterpret_cast<intptr_t>(p) - reinterpret_cast<intptr_t>(base);
  return d < 0 ? -1 : (int64_t)(d / 2);
}

extern "C" int rb_nvfp4_swiglu_forward_strided(const void* gate, const void* up, int64_t ld, int64_t blk,
                                               int64_t rows, int64_t hidden, void* h, int64_t ldh, float* gs_out,
                                               void* workspace, void* stream) {
  rb::SwigluArgs a = {};
  a.gate = reinterpret_cast<const uint16_t*>(gate);
  a.du = (gate == nullptr || up == nullptr || swiglu_misaligned(up)) ? -1 : elem_offset(gate, up);
  a.ld = ld;
  a.blk = blk;
  a.h = reinterpret_cast<uint16_t*>(h);
  a.ldh = ldh;
  a.rows = rows;
  a.hidden = hidden;
  a.gs_out = gs_out;
  return swiglu_launch<false>(a, "nvfp4 swiglu_forward", workspace, stream);
}

extern "C" int rb_nvfp4_swiglu_backward_strided(const void* grad_h, int64_t ldgh, const void* gate, const void* up,
                                                int64_t ld, int64_t blk, int64_t rows, int64_t hidden,
                                                void* grad_gate, void* grad_up, int64_t ldo, int64_t blko,
                                                float* gs_out, void* workspace, void* stream) {
  rb::SwigluArgs a = {};
  a.gate = reinterpret_cast<const uint16_t*>(gate);
  a.du = (gate == nullptr || up == nullptr || swiglu_misaligned(up)) ? -1 : elem_offset(gate, up);
  a.ld = ld;
  a.blk = blk;
  a.grad_h = reinterpret_cast<const uint16_t*>(grad_h);
  a.ldh = ldgh;
  a.grad_gate = reinterpret_cast<uint16_t*>(grad_gate);
  a.dug = (grad_gate == nullptr || grad_up == nullptr || swiglu_misaligned(grad_up)) ? -1
                                                                                      : elem_offset(grad_gate, grad_up);
  a.ldo = ldo;
  a.blko = blko;
  a.rows = rows;
  a.hidden = hidden;
  a.gs_out = gs_out;
  return swiglu_launch<true>(a, "nvfp4 swiglu_backward", workspace, stream);
}
