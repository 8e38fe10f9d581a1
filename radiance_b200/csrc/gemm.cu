// Block-scaled NVFP4 GEMM for B200 on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   out[i, j] = alpha * sum_k (e2m1(a[i,k]) * e4m3(sa[i, k/16])) * (e2m1(b[j,k]) * e4m3(sb[j, k/16])) (+ bias[j])
//
// Replaces torch._scaled_mm_v2 (cuBLASLt) behind radiance's nvfp4_mm/mm
// (src/radiance/nvfp4/quantize.py:359-409), with the global-scale fold, bias add and output cast
// of quantize.py:408-409 and linear.py:82-83 fused into the epilogue.
//
// Design: one persistent CTA per SM, 6 warps, warp-specialised.
//   warp 0 (one lane)  : producer.  Per 256-element K step it TMA-loads the A tile (128 rows x
//                        128 B, 128-byte swizzle), the B tile (256 rows x 128 B) and, with plain
//                        bulk copies, the matching e4m3 scale atoms.  The scale layout written by
//                        the quantizer (SWIZZLE_32_4_4: one 512-byte atom per 128 rows x 4 scale
//                        columns) is exactly what tcgen05.cp.32x128b.warpx4 moves into tensor
//                        memory, so scales go global -> shared -> TMEM untouched.
//   warp 1 (one lane)  : MMA issuer.  Per 64-wide K block, tcgen05.cp of its scale atoms and one
//                        tcgen05.mma.kind::mxf4nvf4.block_scale.scale_vec::4X (128 x 256 x 64) into
//                        a TMEM accumulator; tcgen05.commit frees the smem stage.
//   warps 2-5          : epilogue.  tcgen05.ld the accumulator (each warp owns 32 TMEM lanes =
//                        32 output rows), alpha = ga * gb and bias applied in fp32, one rounding to
//                        bf16 or fp32, staged in swizzled shared memory and written by TMA stores.
// The two accumulator buffers share TMEM columns: buffer 0 is columns [0, 256), buffer 1 is
// [192, 448), and the scale factors live in [448, 512).  The epilogue drains the shared 64
// columns first and releases them, so the next tile's MMAs start while the rest drains.
// No TMA multicast is used (the same kernel serves multi-GPU jobs).
#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

namespace rb {

__device__ uint32_t g_gemm_status;

constexpr int kBM = 128;            // tile rows (M) = TMEM lanes
constexpr int kBN = 256;            // tile cols (N)
constexpr int kStepBytes = 128;     // packed bytes of one K step (256 e2m1 values)
constexpr int kStages = 3;
constexpr int kOverlap = 64;        // TMEM columns shared by the two accumulator buffers
constexpr int kAcc1Col = kBN - kOverlap;   // 192
constexpr int kSfaCol = 512 - kOverlap;    // 448: 4 columns per 64-wide K block (16 total)
constexpr int kSfbCol = kSfaCol + 16;      // 464: 8 columns per K block (32 total)
constexpr int kGemmThreads = 192;
constexpr int kEpiChunk = 64;       // accumulator columns per epilogue step
constexpr int kGroupM = 8;          // raster: tiles visited in groups of 8 M-tiles

struct GemmSmem {
  uint8_t a[kStages][kBM * kStepBytes];   // 16 KB per stage
  uint8_t b[kStages][kBN * kStepBytes];   // 32 KB per stage
  uint8_t sfa[kStages][4 * 512];          // 4 K-blocks x one 128-row atom
  uint8_t sfb[kStages][8 * 512];          // [row half h][K-block kb] at (4h + kb) * 512
  uint8_t out[4][2][4096];                // per epilogue warp: two staged output boxes
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint64_t acc_empty;
  uint64_t drain;
  uint32_t tmem_base;
};

struct GemmArgs {
  int64_t M, N, K;
  const uint8_t* a_scale;
  const uint8_t* b_scale;
  const float* alpha_a;
  const float* alpha_b;
  const void* bias;
  int bias_f32;
  void* out;
  int out_f32;
  int64_t ldo;
  int tiles_m, tiles_n, n_tiles;
  int k_steps, k_blocks;   // K/256 rounded up, K/64
  // Grouped mode (two-SM kernel only): `groups` holds num_groups device records
  // {a_row0, b_row0, out_row0, m, k0, k}; group g computes
  //   out[out_row0 + i, j] = alpha_a[g] alpha_b[g] sum_{k0 <= c < k0 + k} A[a_row0 + i, c] B[b_row0 + j, c]
  // for i < m, j < N.  A and B share one contraction axis of kb_total 64-wide blocks (their scale
  // grids are kb_total blocks wide); out has out_rows rows.
  const int64_t* groups;
  int num_groups;
  int kb_total;
  int64_t out_rows;
  // N-split all-gather fused into the epilogue: npeers device pointers into other GPUs' copies of
  // the output (peer memory mapped into this process), each at the position `out` has in its
  // own; every element stored to `out` is also written to each of them.
  void* peer_out[7];
  int npeers;
  // SwiGLU epilogue (the kernels' kSwiglu instantiation; bf16 output, no peers).  Each 64-column
  // chunk of the output holds [32 gate | 32 up] columns of the same 32 hidden units; besides the
  // output itself the epilogue writes h = silu(g) * u (bf16) at h + row * ldh + col / 2 and folds
  // max |h| into h_ws[0]; the last epilogue warp to finish turns it into the global scale of h.
  void* h;
  int64_t ldh;
  uint32_t* h_ws;  // {max |h| as bf16 bits, finished epilogue warps}: zero on entry, left zero
  float* h_gs;
};

constexpr int kMaxPeers = 7;
constexpr int kMaxGroups = 256;
constexpr int kGroupFields = 6;

// ---------------------------------------------------------------------------------------------
// tcgen05 wrappers (inline PTX)
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_cp_scale(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

#define RB_TMEM_LD_X32(taddr, r)                                                                              \
  asm volatile(                                                                                               \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "  \
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"      \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),       \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),             \
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),             \
        "=r"(r[30]), "=r"(r[31])                                                                              \
      : "r"(taddr))

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major with 128-byte swizzle: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Descriptor of one 512-byte scale atom (32 rows x 16 B, no swizzle, 8-row groups 128 B apart).
__device__ __forceinline__ uint64_t sdesc_scale(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(128 >> 4) << 32) |
         ((uint64_t)1 << 46);
}
// Instruction descriptor: kind::mxf4nvf4, A = B = e2m1 (packed), K-major, ue4m3 scales, M = 128.
__host__ __device__ constexpr uint32_t idesc_nvf4(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& mt, int& nt) {
  const int group = t / (kGroupM * tiles_n);
  const int first_m = group * kGroupM;
  const int gm = min(tiles_m - first_m, kGroupM);
  const int r = t - group * kGroupM * tiles_n;
  mt = first_m + r % gm;
  nt = r / gm;
}

// Waits with the whole warp and returns a warp-uniform result (false after the ~1 s limit).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xFFFFFFFFu, mbar_wait(bar, parity));
}

// The producer's and MMA issuer's waits.  In the SwiGLU instantiation the epilogue bounds the
// kernel and these warps mostly wait for it; they poll with a short sleep so that their polling
// does not take issue slots from the epilogue warps on their schedulers.
template <bool kSwiglu>
__device__ __forceinline__ bool pipe_wait_warp(uint64_t* bar, uint32_t parity) {
  if constexpr (kSwiglu) return __all_sync(0xFFFFFFFFu, mbar_wait_sleep(bar, parity, 32));
  else return mbar_wait_warp(bar, parity);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// The output is written once and not read again by this kernel, so its lines are marked to leave
// L2 first: the operand tiles that later tiles re-read stay resident.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                   map),
               "r"(smem_src), "r"(x), "r"(y), "l"(policy_evict_first())
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N committed bulk groups of this thread still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr int kOutBox = 4096;  // one staged output box: 32 rows x 128 B

// One 32-row x 64-column piece of the output: this warp's 32 accumulator lanes (one output row per
// lane), times alpha, plus bias, rounded once to the output type.  The rows are staged in shared
// memory in the 128-byte-swizzled layout of the output tensor map (16-byte chunk c of row r at
// r * 128 + (c ^ (r % 8)) * 16, which also makes the 32 lanes' writes bank-conflict free) and
// written by one TMA store, so the global write is a few full-line bursts instead of 32 rows of
// scattered 16-byte stores.  `slots` is the warp's two staged boxes (8 KB, 1024-byte aligned):
// bf16 pieces alternate between them, fp32 pieces (two boxes of 32 columns) use both.  Rows at or
// past row_end (the upper half of a 256-row tile when M % 256 == 128, or past a group's end) are
// not stored.
// silu(g) = g / (1 + exp(-g)) with the IEEE fp32 quotient, as torch's silu kernel evaluates it.
__device__ __forceinline__ float silu_ieee(float g) { return g / (1.0f + expf(-g)); }

// silu(g) rounded to bf16, for a bf16 g, is a function of g's 16 bits, and most of them are easy:
//   |g| < 2^-9 (biased exponent e < 118): d = 1 + exp(-g) is within |g| of 2, so g / d is within a
//       relative |g| / 2 < 2^-10 of g / 2, which is a bf16 value (or half of a subnormal one,
//       rounded the same way) -- the result is bf16(g / 2);
//   g >= 128 (e >= 134): exp(-g) is far below half an ulp of 1, d = 1 and the result is g;
//   +inf and NaN: g as well;  g <= -128 (and -inf): evaluated with silu_ieee (the warp takes that
//       path together);
//   the 4096 others (e in 118..133, both signs): a table of bf16 results built with silu_ieee.
// The table replaces an exp, a division and their range handling per element (about 40
// instructions), which the epilogue's one warp per scheduler could not hide behind the MMAs.
// rb_nvfp4_selftest_silu compares the whole mapping with bf16(silu_ieee(g)) for all 65536 g.
constexpr uint32_t kSiluE0 = 118;  // table exponents [kSiluE0, kSiluE0 + 16)
constexpr int kSiluTab = 2048;                     // entries per sign: 16 exponents x 128 significands

// Fills the table at `tab` (threads tid = 0..nthreads-1 of the caller): entry s * 2048 + i is the
// bf16 result for the g with sign s, exponent kSiluE0 + i / 128 and significand i % 128.
__device__ __forceinline__ void silu_table_build(uint32_t tab, int tid, int nthreads) {
  for (int t = tid; t < 2 * kSiluTab; t += nthreads) {
    const uint32_t sgn = (uint32_t)t / kSiluTab, i = (uint32_t)t % kSiluTab;
    const uint32_t b = (sgn << 15) | ((kSiluE0 + (i >> 7)) << 7) | (i & 127u);
    const __nv_bfloat16 r = __float2bfloat16_rn(silu_ieee(__uint_as_float(b << 16)));
    const uint16_t rb = *reinterpret_cast<const uint16_t*>(&r);
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(tab + 2 * (uint32_t)t), "h"(rb) : "memory");
  }
}

// silu(g) as a float holding a bf16 value, for a bf16 g (bits b, value gf) above -128 (finite or
// not: +-inf and NaN above the table range give g itself, as the IEEE evaluation does for +inf and
// NaN).  One table read and two selects; rb_nvfp4_selftest_silu checks it on every bf16 input.
__device__ __forceinline__ float silu_lookup(uint32_t b, float gf, uint32_t tab) {
  const uint32_t idx = ((b - (kSiluE0 << 7)) & 0x7FFu) | ((b >> 4) & 0x800u);  // any valid entry
  uint16_t tv;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(tv) : "r"(tab + 2 * idx));
  const float a = fabsf(gf);
  const float half = __bfloat162float(__float2bfloat16_rn(gf * 0.5f));
  const float t = __uint_as_float((uint32_t)tv << 16);
  return a < 0.001953125f /* 2^-9 */ ? half : (a < 128.0f ? t : gf);  // NaN fails a < 128: gf
}

// silu_lookup for the two bf16 gates in the halves of gw, as a bf16x2 word: the same mapping with
// packed integer and bf16x2 operations.  Per half: |g| < 2^-9 (bits below 0x3B00) gives g * 0.5 as
// one bf16 multiply (the exact product rounded once, as bf16(float(g) * 0.5f) rounds it); bits
// 0x3B00 .. 0x42FF the table entry; |g| >= 128, inf and NaN (bits 0x4300 and up) g itself.
// rb_nvfp4_selftest_silu checks it on every bf16 input in both halves.
__device__ __forceinline__ uint32_t sign_mask2(uint32_t x) {  // 0xFFFF in each half whose bit 15 is set
  uint32_t m;
  asm("prmt.b32 %0, %1, 0, 0xBB99;" : "=r"(m) : "r"(x));
  return m;
}
__device__ __forceinline__ uint32_t silu_lookup2(uint32_t gw, uint32_t tab) {
  const uint32_t a = (gw & 0x7FFF7FFFu) | 0x80008000u;  // |g| bits with a guard bit: no borrow between halves
  const uint32_t not_small = sign_mask2(a - 0x3B003B00u);        // |g| >= 2^-9
  const uint32_t big = sign_mask2(a - 0x43004300u);              // |g| >= 128, inf, NaN
  // Table offsets 2 * (((b - (kSiluE0 << 7)) & 0x7FF) | (sign << 11)) per half; the guard bit in the
  // low half keeps its subtraction from borrowing out of the high half.
  const uint32_t off = ((((gw | 0x8000u) - (kSiluE0 << 7) * 0x10001u) & 0x07FF07FFu) | ((gw >> 4) & 0x08000800u)) << 1;
  uint16_t t0, t1;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(t0) : "r"(tab + (off & 0xFFFFu)));
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(t1) : "r"(tab + (off >> 16)));
  const uint32_t t = (uint32_t)t0 | ((uint32_t)t1 << 16);
  const __nv_bfloat162 hv = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&gw), __float2bfloat162_rn(0.5f));
  const uint32_t halfw = *reinterpret_cast<const uint32_t*>(&hv);
  const uint32_t mid = (t & not_small) | (halfw & ~not_small);
  return (gw & big) | (mid & ~big);
}

// The SwiGLU half of a 64-column piece: v[j] (gate) and v[32 + j] (up), j < 32, are one row's
// pre-activations of 32 consecutive hidden units.  Each h is rounded as radiance's bf16
// F.silu(g) * u rounds it (src/radiance/model/ffn.py:32): g and u to bf16 (as stored in the
// output), silu(g) to bf16, the product (exact in fp32) to bf16.  w receives the row's 32 values
// (one 64-byte run of h); rows at or past row_end are not counted in the maximum.  The whole warp
// runs this: a gate value at or below -128 anywhere in it sends the warp down the IEEE evaluation
// (rare).
__device__ __forceinline__ void swiglu_piece(const float* v, int64_t row, int64_t row_end, uint32_t& hmax,
                                             uint32_t tab, uint32_t (&w)[16]) {
  uint32_t gw[16];
  __nv_bfloat162 mn = __float2bfloat162_rn(0.0f);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    gw[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
    mn = __hmin2(mn, *reinterpret_cast<const __nv_bfloat162*>(&gw[j]));
  }
  const bool far = fminf(__low2float(mn), __high2float(mn)) <= -128.0f;
  if (__any_sync(0xFFFFFFFFu, far)) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float s0 = __bfloat162float(__float2bfloat16_rn(silu_ieee(__uint_as_float(gw[j] << 16))));
      const float s1 = __bfloat162float(__float2bfloat16_rn(silu_ieee(__uint_as_float(gw[j] & 0xFFFF0000u))));
      const uint32_t uw = pack_bf16x2(v[32 + 2 * j], v[32 + 2 * j + 1]);
      w[j] = pack_bf16x2(s0 * __uint_as_float(uw << 16), s1 * __uint_as_float(uw & 0xFFFF0000u));
    }
  } else {
    // silu(g) * u on bf16x2 pairs: the product of two bf16 values is exact in fp32, so one bf16
    // multiply rounds it exactly as the fp32 product rounded to bf16.
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t sw = silu_lookup2(gw[j], tab);
      const __nv_bfloat162 u2 = __floats2bfloat162_rn(v[32 + 2 * j], v[32 + 2 * j + 1]);
      const __nv_bfloat162 h2 = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&sw), u2);
      w[j] = *reinterpret_cast<const uint32_t*>(&h2);
    }
  }
  if (row >= row_end) return;
  uint32_t m2 = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) m2 = __vmaxu2(m2, w[j] & 0x7FFF7FFFu);  // |h| as bf16 bits (NaN above inf)
  hmax = max(hmax, max(m2 & 0xFFFFu, m2 >> 16));
}

// Compares the epilogue's silu (silu_lookup and silu_lookup2 in both halves, and the IEEE
// evaluation at or below -128) with bf16(silu_ieee(g)) on all 65536 bf16 inputs: mismatches[0] counts bf16 results that differ (NaNs
// compare equal), mismatches[1] keeps the largest failing bit pattern plus one.
__global__ void __launch_bounds__(256) selftest_silu_kernel(uint32_t* mismatches) {
  __shared__ __align__(16) uint16_t tab[2 * kSiluTab];
  const uint32_t tab_addr = smem_u32(tab);
  silu_table_build(tab_addr, threadIdx.x, blockDim.x);
  __syncthreads();
  for (uint32_t b = blockIdx.x * blockDim.x + threadIdx.x; b < 65536u; b += gridDim.x * blockDim.x) {
    const float gf = __uint_as_float(b << 16);
    const __nv_bfloat16 r = __float2bfloat16_rn(silu_ieee(gf));
    const uint32_t want = *reinterpret_cast<const uint16_t*>(&r);
    const float sv = gf <= -128.0f ? __bfloat162float(r) : silu_lookup(b, gf, tab_addr);
    // The packed form, with b in the low half next to another gate above -128 in the high half,
    // and in the high half next to that gate.
    const uint32_t o = (b * 40503u + 12345u) & 0x7FFFu;
    const uint32_t lo2 = silu_lookup2(b | (o << 16), tab_addr) & 0xFFFFu;
    const uint32_t hi2 = silu_lookup2(o | (b << 16), tab_addr) >> 16;
    const uint32_t got = __float_as_uint(sv) >> 16;
    const bool nan_w = (want & 0x7FFFu) > 0x7F80u;
    const auto differs = [&](uint32_t x) { return x != want && !(nan_w && (x & 0x7FFFu) > 0x7F80u); };
    if (differs(got) || (gf > -128.0f && (differs(lo2) || differs(hi2)))) {
      atomicAdd(&mismatches[0], 1u);
      atomicMax(&mismatches[1], b + 1u);
    }
  }
}

// End of an epilogue warp's work in SwiGLU mode: fold the warp's max |h| into the workspace; the
// last of the launch's `n_warps` epilogue warps converts it to the global scale of h
// (max(amax / 2688, 1e-12), quantize.py:205-213, NaN passing through) and re-zeroes the workspace.
__device__ __forceinline__ void swiglu_finish(const GemmArgs& g, uint32_t hmax, uint32_t n_warps, int lane) {
  const uint32_t m = __reduce_max_sync(0xFFFFFFFFu, hmax);
  if (lane == 0) {
    atomicMax(&g.h_ws[0], m);
    __threadfence();
    if (atomicAdd(&g.h_ws[1], 1u) == n_warps - 1) {
      __threadfence();
      const uint32_t mb = atomicExch(&g.h_ws[0], 0u) << 16;
      atomicExch(&g.h_ws[1], 0u);
      float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);
      gs = (gs < 1e-12f) ? 1e-12f : gs;
      *g.h_gs = gs;
    }
  }
}

// kOneBox (SwiGLU mode): the warp stages every bf16 piece through the one box at `slots`;
// otherwise bf16 pieces alternate between the warp's two boxes.
//
// kHStage (SwiGLU mode): the piece's h (32 rows x 64 bytes) is staged in the warp's 2 KB box at
// `hbox`, 64-byte swizzled (16-byte chunk c of row r at r * 64 + (c ^ ((r / 2) % 4)) * 16: the
// layout of the h tensor map, and bank-conflict free for the 32 lanes' writes), and written by one
// TMA store with the output box; otherwise each lane stores its row's 64 bytes of h directly.
template <bool kSwiglu, bool kOneBox = kSwiglu, bool kHStage = false>
__device__ __forceinline__ void epilogue_piece(const uint32_t (&r)[kEpiChunk], float alpha, const GemmArgs& g,
                                               const CUtensorMap* tmO, uint32_t slots, int& slot, int col0,
                                               int64_t row0, int64_t row_end, int lane, uint32_t& hmax,
                                               uint32_t tab, const CUtensorMap* tmH = nullptr,
                                               uint32_t hbox = 0) {
  float v[kEpiChunk];
#pragma unroll
  for (int j = 0; j < kEpiChunk; ++j) v[j] = __fmul_rn(__uint_as_float(r[j]), alpha);
  if (g.bias != nullptr) {
    if (g.bias_f32) {
      const float4* bp = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(g.bias) + col0);
#pragma unroll
      for (int j = 0; j < kEpiChunk / 4; ++j) {
        const float4 b = __ldg(bp + j);
        v[4 * j] = __fadd_rn(v[4 * j], b.x);
        v[4 * j + 1] = __fadd_rn(v[4 * j + 1], b.y);
        v[4 * j + 2] = __fadd_rn(v[4 * j + 2], b.z);
        v[4 * j + 3] = __fadd_rn(v[4 * j + 3], b.w);
      }
    } else {
      const uint4* bp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(g.bias) + col0);
#pragma unroll
      for (int j = 0; j < kEpiChunk / 8; ++j) {
        const uint4 b = __ldg(bp + j);
        const uint32_t w[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          v[8 * j + 2 * h] = __fadd_rn(v[8 * j + 2 * h], __uint_as_float(w[h] << 16));
          v[8 * j + 2 * h + 1] = __fadd_rn(v[8 * j + 2 * h + 1], __uint_as_float(w[h] & 0xFFFF0000u));
        }
      }
    }
  }
  uint32_t hw[16];
  if constexpr (kSwiglu) {
    swiglu_piece(v, row0 + lane, row_end, hmax, tab, hw);
    if constexpr (!kHStage) {
      if (row0 + lane < row_end) {
        uint8_t* p = reinterpret_cast<uint8_t*>(g.h) + ((row0 + lane) * g.ldh + (col0 >> 1)) * 2;
#pragma unroll
        for (int q = 0; q < 4; ++q) st_global_v4(p + 16 * q, hw[4 * q], hw[4 * q + 1], hw[4 * q + 2], hw[4 * q + 3]);
      }
    }
  }
  const bool store = row0 < row_end;
  const uint32_t row_off = (uint32_t)lane * 128u, sw = (uint32_t)(lane & 7);
  // Copies a staged box (32 rows x 128 B) to every peer output with coalesced 16-byte stores:
  // lane l moves chunk l % 8 of rows 4i + l/8.  The loads from the box finish before the warp's
  // next __syncwarp, so the box can be refilled right after.
  auto to_peers = [&](uint32_t boxa, int64_t col_bytes) {
    const int esz = g.out_f32 ? 4 : 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = 4 * i + (lane >> 3), c = lane & 7;
      if (row0 + r >= row_end) continue;
      const uint4 val = ld_shared_v4(boxa + r * 128 + ((c ^ (r & 7)) << 4));
      const int64_t off = ((row0 + r) * g.ldo) * esz + col_bytes + c * 16;
      for (int p = 0; p < g.npeers; ++p)
        st_global_v4(reinterpret_cast<uint8_t*>(g.peer_out[p]) + off, val.x, val.y, val.z, val.w);
    }
  };
  if (g.out_f32) {
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        st_shared_v4(slots + h * kOutBox + row_off + ((c ^ sw) << 4), __float_as_uint(v[32 * h + 4 * c]),
                     __float_as_uint(v[32 * h + 4 * c + 1]), __float_as_uint(v[32 * h + 4 * c + 2]),
                     __float_as_uint(v[32 * h + 4 * c + 3]));
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && store) {
      tma_store_2d(tmO, slots, col0, (int)row0);
      tma_store_2d(tmO, slots + kOutBox, col0 + 32, (int)row0);
      bulk_commit_group();
    }
    if (g.npeers > 0 && store) {
      to_peers(slots, (int64_t)col0 * 4);
      to_peers(slots + kOutBox, (int64_t)(col0 + 32) * 4);
    }
  } else {
    if (lane == 0) {
      if constexpr (kOneBox) bulk_wait_read<0>();
      else bulk_wait_read<1>();
    }
    __syncwarp();
    const uint32_t box = kOneBox ? slots : slots + (uint32_t)slot * kOutBox;
    const uint32_t hb = kOneBox ? hbox : hbox + (uint32_t)slot * 2048u;  // kHStage: this piece's h box
#pragma unroll
    for (int c = 0; c < 8; ++c)
      st_shared_v4(box + row_off + ((c ^ sw) << 4), pack_bf16x2(v[8 * c], v[8 * c + 1]),
                   pack_bf16x2(v[8 * c + 2], v[8 * c + 3]), pack_bf16x2(v[8 * c + 4], v[8 * c + 5]),
                   pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
    if constexpr (kHStage) {
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(hb + (uint32_t)lane * 64u + ((uint32_t)(c ^ ((lane >> 1) & 3)) << 4), hw[4 * c], hw[4 * c + 1],
                     hw[4 * c + 2], hw[4 * c + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && store) {
      tma_store_2d(tmO, box, col0, (int)row0);
      if constexpr (kHStage) tma_store_2d(tmH, hb, col0 >> 1, (int)row0);
      bulk_commit_group();
    }
    if (g.npeers > 0 && store) to_peers(box, (int64_t)col0 * 2);
    slot ^= 1;
  }
}

// ---------------------------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------------------------
template <bool kSwiglu>
__global__ void __launch_bounds__(kGemmThreads, 1)
    nvfp4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmO, const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  GemmSmem& sm = *reinterpret_cast<GemmSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.acc_empty, 4);
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    prefetch_tensormap(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // A 512-column allocation is all of the SM's tensor memory, so it starts at address 0.  Using
  // the constant (with every descriptor derived from constants and the stage index) keeps the
  // operands of the tcgen05 instructions in uniform registers, which the issue rate depends on.
  // An allocation anywhere else is reported (status 6) and the CTA computes nothing.
  constexpr uint32_t tmem = 0;
  const bool tmem_ok = sm.tmem_base == 0;
  if (!tmem_ok && threadIdx.x == 0) record_status(&g_gemm_status, kStatusTmemBase);
  const int n_my = (tmem_ok && (int)blockIdx.x < g.n_tiles)
                       ? (g.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    // The whole warp runs the loop (warp-uniform operands); one elected lane issues the copies.
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        int mt, nt;
        tile_coords((int)blockIdx.x + i * (int)gridDim.x, g.tiles_m, g.tiles_n, mt, nt);
        const bool two_halves = (int64_t)nt * kBN + 128 < g.N;
        for (int ks = 0; ks < g.k_steps; ++ks) {
          if (!pipe_wait_warp<kSwiglu>(&sm.empty[stage], phase ^ 1u)) {
            if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          const int nkb = min(4, g.k_blocks - 4 * ks);
          const uint32_t sf_bytes = (uint32_t)nkb * 512u;
          if (elect_one()) {
            mbar_arrive_expect_tx(&sm.full[stage],
                                  kBM * kStepBytes + kBN * kStepBytes + sf_bytes * (two_halves ? 3u : 2u));
            tma_load_2d(sm.a[stage], &tmA, &sm.full[stage], ks * kStepBytes, mt * kBM);
            tma_load_2d(sm.b[stage], &tmB, &sm.full[stage], ks * kStepBytes, nt * kBN);
            bulk_load(sm.sfa[stage], g.a_scale + ((int64_t)mt * g.k_blocks + 4 * ks) * 512, sf_bytes,
                      &sm.full[stage]);
            bulk_load(sm.sfb[stage], g.b_scale + ((int64_t)(2 * nt) * g.k_blocks + 4 * ks) * 512, sf_bytes,
                      &sm.full[stage]);
            if (two_halves)
              bulk_load(sm.sfb[stage] + 4 * 512, g.b_scale + ((int64_t)(2 * nt + 1) * g.k_blocks + 4 * ks) * 512,
                        sf_bytes, &sm.full[stage]);
          }
          __syncwarp();
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop so descriptors stay warp-uniform; one elected lane issues the
    // tcgen05 instructions (issuing them from a one-lane branch costs ~75 cycles each).
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t ad0 = sdesc_sw128(smem_u32(sm.a[0])), bd0 = sdesc_sw128(smem_u32(sm.b[0]));
      const uint64_t sad0 = sdesc_scale(smem_u32(sm.sfa[0])), sbd0 = sdesc_scale(smem_u32(sm.sfb[0]));
      for (int i = 0; i < n_my && ok; ++i) {
        int mt, nt;
        tile_coords((int)blockIdx.x + i * (int)gridDim.x, g.tiles_m, g.tiles_n, mt, nt);
        const int width = (int)min((int64_t)kBN, g.N - (int64_t)nt * kBN);
        const uint32_t idesc = idesc_nvf4(width);
        const uint32_t acc = tmem + ((i & 1) ? kAcc1Col : 0);
        for (int ks = 0; ks < g.k_steps; ++ks) {
          // The TMA bytes are visible to the tensor core once the barrier completes (both are
          // async-proxy accesses ordered by the mbarrier); no tcgen05 fence is needed here.
          if (!mbar_wait_warp(&sm.full[stage], phase)) {
            if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutTma);
            ok = false;
            break;
          }
          const int nkb = min(4, g.k_blocks - 4 * ks);
          // Descriptors of this stage: the address field holds bytes >> 4.
          const uint64_t ad = ad0 + (uint64_t)(stage * ((kBM * kStepBytes) >> 4));
          const uint64_t bd = bd0 + (uint64_t)(stage * ((kBN * kStepBytes) >> 4));
          const uint64_t sad = sad0 + (uint64_t)(stage * ((4 * 512) >> 4));
          const uint64_t sbd = sbd0 + (uint64_t)(stage * ((8 * 512) >> 4));
          if (ks == 0 && i >= 1) {
            if (!pipe_wait_warp<kSwiglu>(&sm.acc_empty, (uint32_t)((i - 1) & 1))) {
              if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutEpilogue);
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (elect_one()) {
            // An MMA starts only after every scale copy issued before it has landed, so each K
            // block's copies go directly before its own MMA (all copies of a step first costs ~20%,
            // copies one block ahead cost more, not less).
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              if (kb < nkb) {
                tc_cp_scale(tmem + kSfaCol + 4 * kb, sad + 32 * kb);
                tc_cp_scale(tmem + kSfbCol + 8 * kb, sbd + 32 * kb);
                if (width > 128) tc_cp_scale(tmem + kSfbCol + 8 * kb + 4, sbd + 32 * (4 + kb));
                tc_mma_nvf4(acc, ad + 2 * kb, bd + 2 * kb, idesc, tmem + kSfaCol + 4 * kb, tmem + kSfbCol + 8 * kb,
                            (ks > 0 || kb > 0) ? 1u : 0u);
              }
            }
            tc_commit(&sm.empty[stage]);
          }
          __syncwarp();
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok && elect_one()) tc_commit(&sm.acc_full);
        __syncwarp();
      }
      // Every MMA this CTA issued has finished once `drain` completes.
      if (elect_one()) tc_commit(&sm.drain);
      __syncwarp();
      mbar_wait_warp(&sm.drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
    // SwiGLU mode: one box per warp (its first; warp q == 1 its second), the 8 KB from sm.out[0][1]
    // through sm.out[1][0] holding the silu table.
    const uint32_t slots = smem_u32(sm.out[q]) + ((kSwiglu && q == 1) ? (uint32_t)kOutBox : 0u);
    int slot = 0;
    uint32_t hmax = 0;  // SwiGLU mode: this lane's max |h| (bf16 bits)
    const uint32_t tab = smem_u32(sm.out[0][1]);  // SwiGLU mode: 8 KB, through sm.out[1][0]
    if constexpr (kSwiglu) {  // the four epilogue warps (threads 64..191) build the silu table
      silu_table_build(tab, (int)threadIdx.x - 64, 128);
      asm volatile("bar.sync 1, 128;" ::: "memory");
    }
    float alpha = 1.0f;
    if (g.alpha_a != nullptr) alpha = *g.alpha_a;
    if (g.alpha_b != nullptr) alpha = __fmul_rn(alpha, *g.alpha_b);
    for (int i = 0; i < n_my; ++i) {
      int mt, nt;
      tile_coords((int)blockIdx.x + i * (int)gridDim.x, g.tiles_m, g.tiles_n, mt, nt);
      const int width = (int)min((int64_t)kBN, g.N - (int64_t)nt * kBN);
      const int buf = i & 1;
      const int base_col = buf ? kAcc1Col : 0;
      if (!mbar_wait_sleep(&sm.acc_full, (uint32_t)(i & 1), 64)) {
        record_status(&g_gemm_status, kStatusTimeoutMma);
        break;
      }
      tc_fence_after();
      const int nch = width / kEpiChunk;
      // Chunks of this buffer that lie in the shared columns [192, 256) go first.
      const int first = (buf == 0) ? ((width == kBN) ? nch - 1 : -1) : 0;
      if (first < 0 && lane == 0) mbar_arrive(&sm.acc_empty);
      const int64_t row0 = (int64_t)mt * kBM + 32 * q;
      for (int step = 0; step < nch; ++step) {
        const int c = (first < 0) ? step : (step == 0 ? first : (buf == 0 ? step - 1 : step));
        uint32_t r[kEpiChunk];
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(base_col + c * kEpiChunk);
        RB_TMEM_LD_X32(taddr, r);
        RB_TMEM_LD_X32(taddr + 32, (r + 32));
        tmem_ld_wait();
        if (step == 0 && first >= 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.acc_empty);
        }
        epilogue_piece<kSwiglu>(r, alpha, g, &tmO, slots, slot, nt * kBN + c * kEpiChunk, row0, g.M, lane, hmax,
                                tab);
      }
    }
    if constexpr (kSwiglu) swiglu_finish(g, hmax, gridDim.x * 4u, lane);
    // The staged boxes must not be overwritten or freed while a TMA store still reads them.
    if (lane == 0) bulk_wait_all();
    if (g.npeers > 0) __threadfence_system();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(sm.tmem_base, 512);
}


// =============================================================================================
// Two-SM variant: a cluster of two CTAs computes a 256 x 256 tile with tcgen05 cta_group::2.
//
// CTA r of the pair loads A rows [256 mt + 128 r, +128) and B rows [256 nt + 128 r, +128) with
// their scale atoms, plus the scale atoms of all 256 B rows (each CTA's tensor core multiplies
// its 128 rows by the whole B tile).  All loads of both CTAs complete on the leader's (rank 0)
// barrier; the leader alone issues tcgen05.cp / tcgen05.mma with cta_group::2, which read the
// same shared-memory offsets in both CTAs and write the same TMEM columns in both.  The leader's
// commits arrive on both CTAs' barriers (multicast commit), and the peer's epilogue warps release
// the shared accumulator columns on the leader's barrier.  One 256x256x64 MMA and three scale
// copies serve two SMs, half the per-FLOP issue and copy work of the one-SM kernel.  The SwiGLU
// instantiation runs eight epilogue warps (10 warps per CTA) and four operand stages (Gemm2Cfg).
// =============================================================================================
constexpr int kSfStep = 2048;  // one K step's scale atoms for 128 rows (4 x 512 B)

// Per instantiation: the plain GEMM keeps five operand stages and four epilogue warps.  The SwiGLU
// GEMM's epilogue also computes and stores h, so it runs two epilogue warps on each TMEM lane
// quarter -- eight in all, two per scheduler, each taking every other 64-column chunk -- and pays
// for their staging boxes, the h boxes and the silu table with one stage less.  Measured at 16384 x
// 11264 x 2048: four stages with one (output, h) box pair per warp 211 us; three stages 231 us with
// one pair or two.
template <bool kSwiglu>
struct Gemm2Cfg {
  static constexpr int kStages = kSwiglu ? 4 : 5;
  static constexpr int kEpiWarps = kSwiglu ? 8 : 4;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA issuer, epilogue
  static constexpr int kSwBoxes = 1;                    // SwiGLU mode: staged (output, h) box pairs per warp
};

template <bool kSwiglu>
struct Gemm2Smem {
  static constexpr int S = Gemm2Cfg<kSwiglu>::kStages;
  uint8_t a[S][kBM * kStepBytes];  // this CTA's 128 A rows (16 KB)
  uint8_t b[S][kBM * kStepBytes];  // this CTA's 128 of the tile's 256 B rows (16 KB)
  uint8_t sfa[S][kSfStep];         // scale atoms of this CTA's A rows
  uint8_t sfb[S][2 * kSfStep];     // scale atoms of all 256 B rows: [half][k block]
  // Staged output boxes: two per epilogue warp, or kSwBoxes per warp in SwiGLU mode, with as many h
  // boxes.
  uint8_t out[kSwiglu ? Gemm2Cfg<kSwiglu>::kEpiWarps * Gemm2Cfg<kSwiglu>::kSwBoxes : 8][4096];
  uint8_t hbox[kSwiglu ? Gemm2Cfg<kSwiglu>::kEpiWarps * Gemm2Cfg<kSwiglu>::kSwBoxes : 1][kSwiglu ? 2048 : 16];
  uint16_t silu_tab[kSwiglu ? 2 * kSiluTab : 8];        // SwiGLU mode: the silu table
  int tile_prefix[kMaxGroups + 1];  // grouped mode: tiles of groups 0..g-1
  uint64_t full[S];                 // leader: both CTAs' loads of a stage
  uint64_t empty[S];                // each CTA: the leader's MMAs finished with a stage
  uint64_t acc_full;                // each CTA: the accumulator of a tile is complete
  uint64_t acc_empty;               // leader: the pair's epilogue warps are done with the shared columns
  uint64_t drain;
  uint32_t tmem_base;
};

// Dynamic shared memory is the struct plus 1 KB for the 1024-byte alignment; 227 KB per CTA at most.
static_assert(sizeof(Gemm2Smem<false>) + 1024 <= 232448 && sizeof(Gemm2Smem<true>) + 1024 <= 232448,
              "two-SM GEMM shared memory exceeds 227 KB");

constexpr uint32_t kStageBytes2 = 2 * kBM * kStepBytes + 3 * kSfStep;  // per CTA

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrives on the barrier at the same shared-memory offset in each CTA of `mask`.
__device__ __forceinline__ void tc_commit2(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void tc_cp_scale2(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tc_mma_nvf4_2sm(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// TMA tile load into this CTA's shared memory that completes on the leader CTA's barrier.
__device__ __forceinline__ void tma_load_2d_to_leader(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                                      int y) {
  const uint32_t leader_bar = smem_u32(bar) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(leader_bar), "r"(x), "r"(y)
      : "memory");
}
// Arrive on the barrier at the same offset in the leader CTA.
// Arrives on the leader CTA's copy of `bar` without release semantics.  The one use is the peer
// epilogue's "shared accumulator columns read": its tcgen05.ld have completed (tcgen05.wait::ld)
// and been fenced (tcgen05.fence::before_thread_sync) before the arrive, and it orders no memory
// writes.  A release.cluster arrive cost ~670 cycles more per tile on that path, which is the
// hand-off from one tile's last MMA to the next tile's first (about 9% of a K = 2048 GEMM).
__device__ __forceinline__ void mbar_arrive_leader(uint64_t* bar) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(smem_u32(bar)));
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

__host__ __device__ constexpr uint32_t idesc_nvf4_m256(int n) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// One 256 x 256 output tile of the two-SM kernel.
struct Tile2 {
  int64_t arow, brow, orow;  // first A row, B row and output row of the tile
  int64_t row_end;           // output rows at or past this are not stored
  int ncol0, width;          // first output column, columns in the tile (128 or 256)
  int kb0, k_blocks;         // contraction: 64-wide blocks kb0 .. kb0 + k_blocks - 1
  int group;                 // alpha index
};

__device__ __forceinline__ bool group_ok(int64_t a0, int64_t b0, int64_t o0, int64_t m, int64_t k0, int64_t k,
                                         const GemmArgs& g) {
  return a0 >= 0 && b0 >= 0 && o0 >= 0 && m >= 0 && k0 >= 0 && k >= 0 && (a0 & 127) == 0 && (b0 & 127) == 0 &&
         (m & 127) == 0 && (k0 & 63) == 0 && (k & 63) == 0 && k0 + k <= 64 * (int64_t)g.kb_total;
}

__device__ __forceinline__ Tile2 tile2_at(int t, const GemmArgs& g, const int* prefix) {
  Tile2 T;
  int mt, nt;
  if (g.groups == nullptr) {
    tile_coords(t, g.tiles_m, g.tiles_n, mt, nt);
    T.arow = T.orow = (int64_t)mt * 256;
    T.brow = (int64_t)nt * kBN;
    T.row_end = g.M;
    T.kb0 = 0;
    T.k_blocks = g.k_blocks;
    T.group = 0;
  } else {
    int lo = 0, hi = g.num_groups - 1;  // the group whose tile range holds t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t) lo = mid;
      else hi = mid - 1;
    }
    const int64_t* d = g.groups + kGroupFields * lo;
    const int64_t a0 = __ldg(d), b0 = __ldg(d + 1), o0 = __ldg(d + 2), m = __ldg(d + 3), k0 = __ldg(d + 4),
                  k = __ldg(d + 5);
    tile_coords(t - prefix[lo], (int)((m + 255) / 256), g.tiles_n, mt, nt);
    T.arow = a0 + (int64_t)mt * 256;
    T.brow = b0 + (int64_t)nt * kBN;
    T.orow = o0 + (int64_t)mt * 256;
    T.row_end = min(o0 + m, g.out_rows);
    T.kb0 = (int)(k0 >> 6);
    T.k_blocks = (int)(k >> 6);
    T.group = lo;
  }
  T.ncol0 = nt * kBN;
  T.width = (int)min((int64_t)kBN, g.N - (int64_t)T.ncol0);
  return T;
}

template <bool kSwiglu>
__global__ void __launch_bounds__(Gemm2Cfg<kSwiglu>::kThreads, 1)
    nvfp4_gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                       const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmH,
                       const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  using Smem = Gemm2Smem<kSwiglu>;
  constexpr int kS = Gemm2Cfg<kSwiglu>::kStages;
  constexpr int kEW = Gemm2Cfg<kSwiglu>::kEpiWarps;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int cid = (int)cluster_id(), ncl = (int)cluster_count();

  if (g.groups != nullptr && warp == 2) {
    // Tiles per group (ceil(m / 256) x tiles_n; 0 for a group that breaks the contract), scanned.
    int run = 0;
    for (int base = 0; base < g.num_groups; base += 32) {
      const int gi = base + lane;
      int cnt = 0;
      if (gi < g.num_groups) {
        const int64_t* d = g.groups + kGroupFields * gi;
        const int64_t a0 = __ldg(d), b0 = __ldg(d + 1), o0 = __ldg(d + 2), m = __ldg(d + 3), k0 = __ldg(d + 4),
                      k = __ldg(d + 5);
        if (group_ok(a0, b0, o0, m, k0, k, g)) cnt = (int)((m + 255) / 256) * g.tiles_n;
        else record_status(&g_gemm_status, kStatusBadGroup);
      }
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += v;
      }
      if (gi < g.num_groups) sm.tile_prefix[gi + 1] = run + incl;
      run += __shfl_sync(0xFFFFFFFFu, incl, 31);
    }
    if (lane == 0) sm.tile_prefix[0] = 0;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.acc_full, 1);
    mbar_init(&sm.acc_empty, 2 * kEW);
    mbar_init(&sm.drain, 1);
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
    prefetch_tensormap(&tmSA);
    prefetch_tensormap(&tmSB);
    prefetch_tensormap(&tmO);
    if constexpr (kSwiglu) prefetch_tensormap(&tmH);
  }
  if (warp == 1) {
    tmem_alloc2(&sm.tmem_base, 512);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  // A 512-column allocation is all of the SM's tensor memory (the same columns in both CTAs of the
  // pair), so it starts at address 0.  Using the constant (with every descriptor derived from
  // constants and the stage index) keeps the operands of the tcgen05 instructions in uniform
  // registers, which the issue rate depends on (~10% of GEMM throughput).  An allocation anywhere
  // else is reported (status 6) and the pair computes nothing.
  constexpr uint32_t tmem = 0;
  const bool tmem_ok = sm.tmem_base == 0;
  if (!tmem_ok && threadIdx.x == 0) record_status(&g_gemm_status, kStatusTmemBase);
  const int n_tiles = (g.groups == nullptr) ? g.n_tiles : sm.tile_prefix[g.num_groups];
  const int n_my = (tmem_ok && cid < n_tiles) ? (n_tiles - cid + ncl - 1) / ncl : 0;  // 256x256 tiles of this pair

  if (warp == 0) {
    // ------------------------------------------------------------------ producer (both CTAs)
    {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < n_my && ok; ++i) {
        const Tile2 T = tile2_at(cid + i * ncl, g, sm.tile_prefix);
        const int64_t arow = T.arow + (int64_t)rank * kBM;  // this CTA's 128 rows of A
        // Each CTA supplies half of the tile's B rows: 128 for a 256-wide tile, 64 for a 128-wide
        // tail (rows loaded past that half are never read by the MMA).
        const int64_t brow = T.brow + (int64_t)rank * (T.width / 2);
        // Scale atoms: one 256-byte row pair per (128-row tile, 64-wide K block).
        const int64_t sa_row = (arow / kBM) * g.kb_total + T.kb0, sb_row = (T.brow / kBM) * g.kb_total + T.kb0;
        const int k_steps = (T.k_blocks + 3) / 4;
        for (int ks = 0; ks < k_steps; ++ks) {
          if (!pipe_wait_warp<kSwiglu>(&sm.empty[stage], phase ^ 1u)) {
            if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutProducer);
            ok = false;
            break;
          }
          if (elect_one()) {
            const int kx = (T.kb0 + 4 * ks) * 32;  // packed bytes
            if (rank == 0) mbar_arrive_expect_tx(&sm.full[stage], 2 * kStageBytes2);
            tma_load_2d_to_leader(sm.a[stage], &tmA, &sm.full[stage], kx, (int)arow);
            tma_load_2d_to_leader(sm.b[stage], &tmB, &sm.full[stage], kx, (int)brow);
            tma_load_2d_to_leader(sm.sfa[stage], &tmSA, &sm.full[stage], 0, (int)((sa_row + 4 * ks) * 2));
            tma_load_2d_to_leader(sm.sfb[stage], &tmSB, &sm.full[stage], 0, (int)((sb_row + 4 * ks) * 2));
            tma_load_2d_to_leader(sm.sfb[stage] + kSfStep, &tmSB, &sm.full[stage], 0,
                                  (int)((sb_row + g.kb_total + 4 * ks) * 2));
          }
          __syncwarp();
          if (++stage == kS) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader only)
    if (rank == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint64_t ad0 = sdesc_sw128(smem_u32(sm.a[0])), bd0 = sdesc_sw128(smem_u32(sm.b[0]));
      const uint64_t sad0 = sdesc_scale(smem_u32(sm.sfa[0])), sbd0 = sdesc_scale(smem_u32(sm.sfb[0]));
      for (int i = 0; i < n_my && ok; ++i) {
        const Tile2 T = tile2_at(cid + i * ncl, g, sm.tile_prefix);
        const int width = T.width;
        const uint32_t idesc = idesc_nvf4_m256(width);
        const uint32_t acc = tmem + ((i & 1) ? kAcc1Col : 0);
        if (i >= 1) {
          if (!pipe_wait_warp<kSwiglu>(&sm.acc_empty, (uint32_t)((i - 1) & 1))) {
            if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutEpilogue);
            break;
          }
          tc_fence_after();
        }
        const int k_steps = (T.k_blocks + 3) / 4;
        for (int ks = 0; ks < k_steps; ++ks) {
          if (!mbar_wait_warp(&sm.full[stage], phase)) {
            if (lane == 0) record_status(&g_gemm_status, kStatusTimeoutTma);
            ok = false;
            break;
          }
          const int nkb = min(4, T.k_blocks - 4 * ks);
          // Descriptors of this stage: the address field holds bytes >> 4.
          const uint64_t ad = ad0 + (uint64_t)(stage * ((kBM * kStepBytes) >> 4));
          const uint64_t bd = bd0 + (uint64_t)(stage * ((kBM * kStepBytes) >> 4));
          const uint64_t sad = sad0 + (uint64_t)(stage * (kSfStep >> 4));
          const uint64_t sbd = sbd0 + (uint64_t)(stage * ((2 * kSfStep) >> 4));
          if (elect_one()) {
            // As in the one-SM kernel, each K block's scale copies directly precede its MMA.
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
              if (kb < nkb) {
                tc_cp_scale2(tmem + kSfaCol + 4 * kb, sad + 32 * kb);
                tc_cp_scale2(tmem + kSfbCol + 8 * kb, sbd + 32 * kb);
                if (width > 128) tc_cp_scale2(tmem + kSfbCol + 8 * kb + 4, sbd + ((kSfStep + kb * 512) >> 4));
                tc_mma_nvf4_2sm(acc, ad + 2 * kb, bd + 2 * kb, idesc, tmem + kSfaCol + 4 * kb, tmem + kSfbCol + 8 * kb,
                                (ks > 0 || kb > 0) ? 1u : 0u);
              }
            }
            tc_commit2(&sm.empty[stage], 0x3);
          }
          __syncwarp();
          if (++stage == kS) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok && elect_one()) tc_commit2(&sm.acc_full, 0x3);
        __syncwarp();
      }
      // Every MMA of the pair has finished once `drain` completes.
      if (elect_one()) tc_commit2(&sm.drain, 0x1);
      __syncwarp();
      mbar_wait_warp(&sm.drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2 .. 2+kEW-1, both CTAs)
    // A warp reaches the TMEM lanes of its warp id mod 4.  With eight epilogue warps, warps w and
    // w + 4 share a lane quarter and split its 64-column chunks: `half` takes chunks c with
    // c % 2 == half.
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31
    constexpr int kStride = kEW / 4;
    const int half = (warp - 2) / 4;
    // Staging: two boxes per warp (pieces alternate between them), or in SwiGLU mode kSwBoxes
    // (output, h) box pairs per warp.
    constexpr int kBoxes = kSwiglu ? Gemm2Cfg<kSwiglu>::kSwBoxes : 2;
    const uint32_t slots = smem_u32(&sm.out[(kSwiglu ? warp - 2 : q) * kBoxes][0]);
    int slot = 0;
    uint32_t hmax = 0;  // SwiGLU mode: this lane's max |h| (bf16 bits)
    const uint32_t tab = smem_u32(&sm.silu_tab[0]);
    const uint32_t hbox = smem_u32(&sm.hbox[kSwiglu ? (warp - 2) * kBoxes : 0][0]);
    if constexpr (kSwiglu) {  // the epilogue warps (threads 64 ..) build the silu table
      silu_table_build(tab, (int)threadIdx.x - 64, 32 * kEW);
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kEW) : "memory");
    }
    for (int i = 0; i < n_my; ++i) {
      const Tile2 T = tile2_at(cid + i * ncl, g, sm.tile_prefix);
      const int width = T.width;
      float alpha = 1.0f;
      if (g.alpha_a != nullptr) alpha = __ldg(g.alpha_a + T.group);
      if (g.alpha_b != nullptr) alpha = __fmul_rn(alpha, __ldg(g.alpha_b + T.group));
      const int buf = i & 1;
      const int base_col = buf ? kAcc1Col : 0;
      if (!mbar_wait_sleep(&sm.acc_full, (uint32_t)(i & 1), 64)) {
        record_status(&g_gemm_status, kStatusTimeoutMma);
        break;
      }
      tc_fence_after();
      const int nch = width / kEpiChunk;
      // The chunk in the columns both buffers use ([192, 256)): its reader drains it first and then
      // releases; every other warp releases at once.  acc_empty completes after all 2 * kEW.
      const int sc = (buf == 0) ? ((width == kBN) ? nch - 1 : -1) : 0;
      const bool mine_sc = sc >= 0 && (sc % kStride) == half;
      auto release = [&]() {
        if (rank == 0) mbar_arrive(&sm.acc_empty);
        else mbar_arrive_leader(&sm.acc_empty);
      };
      if (!mine_sc && lane == 0) release();
      const int64_t row0 = T.orow + (int64_t)rank * kBM + 32 * q;
      const int nmine = (nch - half + kStride - 1) / kStride;
      for (int step = 0; step < nmine; ++step) {
        // This warp's chunks in ascending order, except that a shared last chunk (buffer 0) goes first.
        const int c = (mine_sc && buf == 0) ? (step == 0 ? sc : half + (step - 1) * kStride) : half + step * kStride;
        uint32_t r[kEpiChunk];
        if (T.k_blocks > 0) {
          const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(base_col + c * kEpiChunk);
          RB_TMEM_LD_X32(taddr, r);
          RB_TMEM_LD_X32(taddr + 32, (r + 32));
          tmem_ld_wait();
        } else {  // an empty contraction: the product is zero (no MMA wrote the accumulator)
#pragma unroll
          for (int j = 0; j < kEpiChunk; ++j) r[j] = 0u;
        }
        if (step == 0 && mine_sc) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release();
        }
        epilogue_piece<kSwiglu, kSwiglu && kBoxes == 1, kSwiglu>(r, alpha, g, &tmO, slots, slot,
                                                                 T.ncol0 + c * kEpiChunk, row0, T.row_end, lane,
                                                                 hmax, tab, &tmH, hbox);
      }
    }
    if constexpr (kSwiglu) swiglu_finish(g, hmax, gridDim.x * (uint32_t)kEW, lane);
    if (lane == 0) bulk_wait_all();
    if (g.npeers > 0) __threadfence_system();
    __syncwarp();
  }

  // Both CTAs stay until every MMA of the pair is done (the leader drained them above), then free
  // the pair's tensor memory together.
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) tmem_dealloc2(sm.tmem_base, 512);
}

}  // namespace rb

// =============================================================================================
// Host entry points
// =============================================================================================
using namespace rb;

namespace {

// Launches the two-SM kernel on min(clusters_wanted, resident clusters) CTA pairs.  A and B scale
// buffers are viewed as rows of 256 bytes (half a 512-byte atom): one K step of one 128-row tile
// is 8 consecutive rows.
template <bool kSwiglu>
int launch_two_sm(GemmArgs& g, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO,
                  const void* a_scale, int64_t a_rows, const void* b_scale, int64_t b_rows, int clusters_wanted,
                  int dev, cudaStream_t st, const CUtensorMap* tmH = nullptr) {
  CUtensorMap tmSA, tmSB;
  if (!rb_host::make_tmap_2d(&tmSA, a_scale, CU_TENSOR_MAP_DATA_TYPE_UINT8, 256,
                             (uint64_t)(a_rows / 128) * (uint64_t)g.kb_total * 2, 256, 256, 8,
                             CU_TENSOR_MAP_SWIZZLE_NONE) ||
      !rb_host::make_tmap_2d(&tmSB, b_scale, CU_TENSOR_MAP_DATA_TYPE_UINT8, 256,
                             (uint64_t)(b_rows / 128) * (uint64_t)g.kb_total * 2, 256, 256, 8,
                             CU_TENSOR_MAP_SWIZZLE_NONE))
    return RB_ERR_CUDA;
  const int sms = rb_host::sm_budget(dev);
  const size_t smem = sizeof(Gemm2Smem<kSwiglu>) + 1024;
  static int max_clusters[64] = {0};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Gemm2Cfg<kSwiglu>::kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dev >= 0 && dev < 64 && max_clusters[dev] == 0) {
    if (cudaFuncSetAttribute(nvfp4_gemm2_kernel<kSwiglu>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      rb_host::set_error("cudaFuncSetAttribute(gemm2) failed: %s", cudaGetErrorString(cudaGetLastError()));
      return RB_ERR_CUDA;
    }
    cfg.gridDim = dim3(2 * (sms / 2), 1, 1);
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, nvfp4_gemm2_kernel<kSwiglu>, &cfg) != cudaSuccess || nc < 1) {
      cudaGetLastError();
      nc = sms / 2;
    }
    max_clusters[dev] = nc;
  }
  const int cap = min((dev >= 0 && dev < 64) ? max_clusters[dev] : sms / 2, sms / 2);
  const int clusters = clusters_wanted < cap ? clusters_wanted : cap;
  if (clusters < 1) return RB_OK;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  // tmH (SwiGLU mode: the h output) is unused by the plain kernel, which gets tmO in its place.
  cudaError_t e = cudaLaunchKernelEx(&cfg, nvfp4_gemm2_kernel<kSwiglu>, tmA, tmB, tmSA, tmSB, tmO,
                                     tmH != nullptr ? *tmH : tmO, g);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 gemm launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

// Launches the one-SM kernel (m < 256) on min(tiles, SMs) CTAs.
template <bool kSwiglu>
int launch_one_sm(const GemmArgs& g, const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmO, int dev,
                  cudaStream_t st) {
  const int sms = rb_host::sm_budget(dev);
  const size_t smem = sizeof(GemmSmem) + 1024;
  static bool configured[64] = {false};
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(nvfp4_gemm_kernel<kSwiglu>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      rb_host::set_error("cudaFuncSetAttribute(gemm) failed: %s", cudaGetErrorString(cudaGetLastError()));
      return RB_ERR_CUDA;
    }
    configured[dev] = true;
  }
  const int grid = g.n_tiles < sms ? g.n_tiles : sms;
  nvfp4_gemm_kernel<kSwiglu><<<grid, kGemmThreads, smem, st>>>(tmA, tmB, tmO, g);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 gemm launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

bool sm100_device(int dev, const char* what) {
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) {
    rb_host::set_error("%s: the current device is not an sm_100 GPU", what);
    return false;
  }
  return true;
}

}  // namespace

namespace rb {
// Failure-path self-test for the GEMM's status word: one CTA waits, the way the epilogue waits for
// an accumulator (sleeping between polls), on an mbarrier that nothing ever arrives on -- no TMA,
// MMA or TMEM allocation is made, so nothing is in flight when it gives up after `limit` cycles.
// It then records kStatusTimeoutMma, as the epilogue does, and returns.
__global__ void gemm_selftest_wait_kernel(long long limit, uint32_t* waited) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const long long t0 = clock64();
  const bool ok = mbar_wait_sleep(&bar, 0, 64, limit);
  const long long t1 = clock64();
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) {
      record_status(&g_gemm_status, kStatusTimeoutMma);
      *waited = (uint32_t)min(t1 - t0, (long long)0xFFFFFFFF);
    }
    return;
  }
}
}  // namespace rb

extern "C" {

uint32_t rb_internal_gemm_selftest_wait(long long limit, uint32_t* waited, cudaStream_t stream) {
  rb::gemm_selftest_wait_kernel<<<1, 128, 0, stream>>>(limit, waited);
  return 0;
}

uint32_t rb_internal_gemm_status(int clear) {
  uint32_t v = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, rb::g_gemm_status, sizeof(v));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(rb::g_gemm_status, &z, sizeof(z));
  }
  return v;
}

// SwiGLU outputs of rb_nvfp4_gemm_swiglu (all null for the plain GEMM).
struct SwigluOut {
  void* h = nullptr;
  int64_t ldh = 0;
  uint32_t* ws = nullptr;
  float* gs = nullptr;
};

static int gemm_impl(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale, int64_t m,
                     int64_t n, int64_t k, const float* alpha_a, const float* alpha_b, const void* bias,
                     int bias_dtype, void* out, int out_dtype, int64_t ldo, void* const* peer_out, int npeers,
                     void* stream, const SwigluOut& sw = SwigluOut()) {
  if (npeers < 0 || npeers > kMaxPeers || (npeers > 0 && peer_out == nullptr)) {
    rb_host::set_error("nvfp4 gemm: npeers must be in [0, %d] with a peer pointer array", kMaxPeers);
    return RB_ERR_ARG;
  }
  for (int p = 0; p < npeers; ++p) {
    if (peer_out[p] == nullptr || (reinterpret_cast<uintptr_t>(peer_out[p]) & 15) != 0) {
      rb_host::set_error("nvfp4 gemm: peer output %d is null or not 16-byte aligned", p);
      return RB_ERR_ARG;
    }
  }
  if (m <= 0 || n <= 0 || k <= 0 || m % 128 != 0 || n % 128 != 0 || k % 64 != 0) {
    rb_host::set_error("nvfp4 gemm needs m %% 128 == 0, n %% 128 == 0 and k %% 64 == 0, got (%lld, %lld, %lld)",
                       (long long)m, (long long)n, (long long)k);
    return RB_ERR_SHAPE;
  }
  if (a_packed == nullptr || a_scale == nullptr || b_packed == nullptr || b_scale == nullptr || out == nullptr) {
    rb_host::set_error("nvfp4 gemm: null pointer argument");
    return RB_ERR_ARG;
  }
  if (out_dtype != RB_OUT_BF16 && out_dtype != RB_OUT_F32) {
    rb_host::set_error("nvfp4 gemm: unsupported output dtype %d", out_dtype);
    return RB_ERR_ARG;
  }
  if (bias != nullptr && bias_dtype != RB_DTYPE_BF16 && bias_dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 gemm: unsupported bias dtype %d", bias_dtype);
    return RB_ERR_ARG;
  }
  const int oesize = out_dtype == RB_OUT_F32 ? 4 : 2;
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(a_packed) || misaligned(b_packed) || misaligned(a_scale) || misaligned(b_scale) || misaligned(out) ||
      (bias != nullptr && misaligned(bias)) || ldo < n || ((uint64_t)ldo * oesize) % 16 != 0) {
    rb_host::set_error("nvfp4 gemm: operands, bias and output must be 16-byte aligned with 16-byte row strides");
    return RB_ERR_ARG;
  }
  const bool swiglu = sw.h != nullptr;
  if (swiglu && (out_dtype != RB_OUT_BF16 || npeers != 0 || n % 64 != 0 || sw.ws == nullptr || sw.gs == nullptr ||
                 misaligned(sw.h) || sw.ldh < n / 2 || ((uint64_t)sw.ldh * 2) % 16 != 0 ||
                 (reinterpret_cast<uintptr_t>(sw.ws) & 7) != 0)) {
    rb_host::set_error("nvfp4 gemm_swiglu: needs a bf16 output, n %% 64 == 0, a 16-byte aligned h with ldh >= n/2 "
                       "and a 16-byte row stride, an 8-byte aligned zeroed workspace and a global-scale pointer");
    return RB_ERR_ARG;
  }
  int dev = rb_host::current_device();
  if (!sm100_device(dev, "nvfp4 gemm")) return RB_ERR_DEVICE;
  GemmArgs g;
  g.h = sw.h;
  g.ldh = sw.ldh;
  g.h_ws = sw.ws;
  g.h_gs = sw.gs;
  g.groups = nullptr;
  g.num_groups = 0;
  g.out_rows = m;
  g.npeers = npeers;
  for (int p = 0; p < kMaxPeers; ++p) g.peer_out[p] = p < npeers ? peer_out[p] : nullptr;
  g.M = m;
  g.N = n;
  g.K = k;
  g.a_scale = reinterpret_cast<const uint8_t*>(a_scale);
  g.b_scale = reinterpret_cast<const uint8_t*>(b_scale);
  g.alpha_a = alpha_a;
  g.alpha_b = alpha_b;
  g.bias = bias;
  g.bias_f32 = bias_dtype == RB_DTYPE_F32;
  g.out = out;
  g.out_f32 = out_dtype == RB_OUT_F32;
  g.ldo = ldo;
  g.k_blocks = (int)(k / 64);
  g.kb_total = g.k_blocks;
  g.k_steps = (g.k_blocks + 3) / 4;
  g.tiles_n = (int)((n + kBN - 1) / kBN);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int sms = rb_host::sm_budget(dev);
  const bool two_sm = m >= 256;
  CUtensorMap tmA, tmB, tmO;
  // Output boxes are 32 rows x 128 bytes (64 bf16 or 32 fp32 columns), 128-byte swizzled.
  if (!rb_host::make_tmap_2d(&tmA, a_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(k / 2), (uint64_t)m,
                             (uint64_t)(k / 2), kStepBytes, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !rb_host::make_tmap_2d(&tmB, b_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(k / 2), (uint64_t)n,
                             (uint64_t)(k / 2), kStepBytes, two_sm ? kBM : kBN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !rb_host::make_tmap_2d(&tmO, out, oesize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             (uint64_t)n, (uint64_t)m, (uint64_t)ldo * oesize, 128 / oesize, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return RB_ERR_CUDA;
  if (two_sm) {
    g.tiles_m = (int)((m + 255) / 256);
    g.n_tiles = g.tiles_m * g.tiles_n;
    if (swiglu) {
      // h boxes: 32 rows x 32 bf16 (64 bytes), 64-byte swizzled; rows past m are clipped.
      CUtensorMap tmH;
      if (!rb_host::make_tmap_2d(&tmH, sw.h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)(n / 2), (uint64_t)m,
                                 (uint64_t)sw.ldh * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return RB_ERR_CUDA;
      return launch_two_sm<true>(g, tmA, tmB, tmO, a_scale, m, b_scale, n, g.n_tiles, dev, st, &tmH);
    }
    return launch_two_sm<false>(g, tmA, tmB, tmO, a_scale, m, b_scale, n, g.n_tiles, dev, st);
  }
  g.tiles_m = (int)(m / kBM);
  g.n_tiles = g.tiles_m * g.tiles_n;
  return swiglu ? launch_one_sm<true>(g, tmA, tmB, tmO, dev, st) : launch_one_sm<false>(g, tmA, tmB, tmO, dev, st);
}

int rb_nvfp4_gemm(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale, int64_t m,
                  int64_t n, int64_t k, const float* alpha_a, const float* alpha_b, const void* bias, int bias_dtype,
                  void* out, int out_dtype, int64_t ldo, void* stream) {
  return gemm_impl(a_packed, a_scale, b_packed, b_scale, m, n, k, alpha_a, alpha_b, bias, bias_dtype, out, out_dtype,
                   ldo, nullptr, 0, stream);
}

int rb_nvfp4_gemm_allgather(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale,
                            int64_t m, int64_t n, int64_t k, const float* alpha_a, const float* alpha_b,
                            const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                            void* const* peer_out, int npeers, void* stream) {
  return gemm_impl(a_packed, a_scale, b_packed, b_scale, m, n, k, alpha_a, alpha_b, bias, bias_dtype, out, out_dtype,
                   ldo, peer_out, npeers, stream);
}

int rb_nvfp4_gemm_swiglu(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale,
                         int64_t m, int64_t n, int64_t k, const float* alpha_a, const float* alpha_b, const void* bias,
                         int bias_dtype, void* out, int64_t ldo, void* h, int64_t ldh, void* workspace,
                         float* h_global_scale, void* stream) {
  if (h == nullptr) {
    rb_host::set_error("nvfp4 gemm_swiglu: null h");
    return RB_ERR_ARG;
  }
  SwigluOut sw;
  sw.h = h;
  sw.ldh = ldh;
  sw.ws = reinterpret_cast<uint32_t*>(workspace);
  sw.gs = h_global_scale;
  return gemm_impl(a_packed, a_scale, b_packed, b_scale, m, n, k, alpha_a, alpha_b, bias, bias_dtype, out,
                   RB_OUT_BF16, ldo, nullptr, 0, stream, sw);
}

int rb_nvfp4_selftest_silu(uint32_t* mismatches, void* stream) {
  if (mismatches == nullptr) {
    rb_host::set_error("nvfp4 selftest_silu: null output");
    return RB_ERR_ARG;
  }
  if (!sm100_device(rb_host::current_device(), "nvfp4 selftest_silu")) return RB_ERR_DEVICE;
  rb::selftest_silu_kernel<<<64, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(mismatches);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("selftest_silu launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_nvfp4_gemm_grouped(const void* a_packed, const void* a_scale, int64_t a_rows, const void* b_packed,
                          const void* b_scale, int64_t b_rows, int64_t n, int64_t k_total, const int64_t* groups,
                          int num_groups, const float* alpha_a, const float* alpha_b, void* out, int out_dtype,
                          int64_t out_rows, int64_t ldo, void* stream) {
  if (a_rows <= 0 || b_rows <= 0 || n <= 0 || k_total <= 0 || out_rows <= 0 || a_rows % 128 != 0 ||
      b_rows % 128 != 0 || n % 128 != 0 || k_total % 64 != 0) {
    rb_host::set_error(
        "nvfp4 grouped gemm needs a_rows %% 128 == 0, b_rows %% 128 == 0, n %% 128 == 0 and k_total %% 64 == 0, "
        "got (%lld, %lld, %lld, %lld)",
        (long long)a_rows, (long long)b_rows, (long long)n, (long long)k_total);
    return RB_ERR_SHAPE;
  }
  if (num_groups < 0 || num_groups > kMaxGroups) {
    rb_host::set_error("nvfp4 grouped gemm: num_groups must be in [0, %d], got %d", kMaxGroups, num_groups);
    return RB_ERR_ARG;
  }
  if (num_groups == 0) return RB_OK;
  if (a_packed == nullptr || a_scale == nullptr || b_packed == nullptr || b_scale == nullptr || out == nullptr ||
      groups == nullptr) {
    rb_host::set_error("nvfp4 grouped gemm: null pointer argument");
    return RB_ERR_ARG;
  }
  if (out_dtype != RB_OUT_BF16 && out_dtype != RB_OUT_F32) {
    rb_host::set_error("nvfp4 grouped gemm: unsupported output dtype %d", out_dtype);
    return RB_ERR_ARG;
  }
  const int oesize = out_dtype == RB_OUT_F32 ? 4 : 2;
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(a_packed) || misaligned(b_packed) || misaligned(a_scale) || misaligned(b_scale) || misaligned(out) ||
      (reinterpret_cast<uintptr_t>(groups) & 7) != 0 || ldo < n || ((uint64_t)ldo * oesize) % 16 != 0) {
    rb_host::set_error("nvfp4 grouped gemm: operands and output must be 16-byte aligned with 16-byte row strides");
    return RB_ERR_ARG;
  }
  if (k_total / 64 > 0x7FFFFFFF / 2 || (a_rows / 128) * (k_total / 64) * 2 > 0x7FFFFFFF ||
      (b_rows / 128) * (k_total / 64) * 2 > 0x7FFFFFFF || a_rows > 0x7FFFFFFF || b_rows > 0x7FFFFFFF ||
      out_rows > 0x7FFFFFFF) {
    rb_host::set_error("nvfp4 grouped gemm: operand too large for 32-bit tensor-map coordinates");
    return RB_ERR_SHAPE;
  }
  int dev = rb_host::current_device();
  if (!sm100_device(dev, "nvfp4 grouped gemm")) return RB_ERR_DEVICE;
  GemmArgs g;
  g.h = nullptr;
  g.ldh = 0;
  g.h_ws = nullptr;
  g.h_gs = nullptr;
  g.M = out_rows;
  g.N = n;
  g.K = k_total;
  g.a_scale = reinterpret_cast<const uint8_t*>(a_scale);
  g.b_scale = reinterpret_cast<const uint8_t*>(b_scale);
  g.alpha_a = alpha_a;
  g.alpha_b = alpha_b;
  g.bias = nullptr;
  g.bias_f32 = 0;
  g.out = out;
  g.out_f32 = out_dtype == RB_OUT_F32;
  g.ldo = ldo;
  g.tiles_m = 0;
  g.tiles_n = (int)((n + kBN - 1) / kBN);
  g.n_tiles = 0;
  g.k_blocks = 0;
  g.k_steps = 0;
  g.groups = groups;
  g.num_groups = num_groups;
  g.kb_total = (int)(k_total / 64);
  g.out_rows = out_rows;
  g.npeers = 0;
  for (int p = 0; p < kMaxPeers; ++p) g.peer_out[p] = nullptr;
  CUtensorMap tmA, tmB, tmO;
  if (!rb_host::make_tmap_2d(&tmA, a_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(k_total / 2), (uint64_t)a_rows,
                             (uint64_t)(k_total / 2), kStepBytes, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !rb_host::make_tmap_2d(&tmB, b_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(k_total / 2), (uint64_t)b_rows,
                             (uint64_t)(k_total / 2), kStepBytes, kBM, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !rb_host::make_tmap_2d(&tmO, out, oesize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             (uint64_t)n, (uint64_t)out_rows, (uint64_t)ldo * oesize, 128 / oesize, 32,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return RB_ERR_CUDA;
  // The group sizes live on the device: every resident cluster starts, reads the table and takes
  // its share of the tiles (clusters without one exit).
  return launch_two_sm<false>(g, tmA, tmB, tmO, a_scale, a_rows, b_scale, b_rows, 1 << 30, dev,
                       reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
