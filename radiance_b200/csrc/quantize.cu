// NVFP4 quantizer and global-scale (amax) kernels for B200 (sm_100a).
//
// Semantics follow radiance's pure-torch emulation, src/radiance/nvfp4/quantize.py:
//   global scale  gs    = max(amax|x| / 2688, 1e-12)                         (:205-213)
//   block scale   s     = clamp(amax_block / (6*gs), 1e-12, 448), rounded UP to e4m3 (:160-202)
//   divisor       D     = e4m3(s) * gs   (one fp32 multiply; 1*gs for an all-zero block)
//   code          q     = RN(x / D), encoded round-to-nearest-even on the e2m1 grid (:93-139)
//   colblock + R  y_i   = sum_j R[j][i] * x_j, j = 0..15 left to right in fp32 (:261-262)
// and the codes/scale bytes are bit-identical to the reference for round-to-nearest.
//
// Design (persistent CTAs, two per SM, 256 threads each):
//   * A 128-row x 128-byte-wide input tile (128 x 128 bf16 or 128 x 64 fp32) is brought into
//     shared memory by TMA as two 128-byte-swizzled boxes, three tiles in flight per CTA.  Every
//     address a thread reads is (a per-tile base) XOR (a constant below 128) plus a constant, so
//     the swizzle costs eight logic ops per tile and the loads take immediate offsets; both walks
//     below are bank-conflict free.
//   * Rowblock form: thread t owns row t % 128 and the 64 (bf16) or 32 (fp32) columns of box
//     t / 128: four or two 16-element blocks, one 4- or 2-byte run of its scale-atom row, and a
//     32- or 16-byte run of its packed row.
//   * Colblock form: a unit is a 16-row group of two adjacent columns, whose two blocks are worked
//     as float2 pairs on Blackwell's packed f32x2 FMA path.  A bf16 thread owns one column pair
//     over 32 rows (two units) and stores each column's 16-byte run of the transposed output and
//     its 2-byte run of scales directly: no staging and no block-wide barrier inside a tile.
//   * x / D is never computed with a divide instruction.  Each block looks up D and
//     Y = RN(1/D) in a 127-entry table (one entry per e4m3 byte, built per CTA with the IEEE
//     reciprocal) and refines q0 = x*Y with two residual corrections r = x - q*D, q += r*Y, each a
//     single fused multiply-add.  That is Markstein's correctly rounded division (P. Markstein,
//     "Computation of elementary functions on the IBM RISC System/6000 processor", IBM J. R&D
//     34(1), 1990; see also Muller et al., Handbook of Floating-Point Arithmetic, ch. 4): after the
//     first correction q is faithful, and a faithful q with a correctly rounded reciprocal gives
//     the correctly rounded quotient after the second.  It holds while the residual x - q*d is a
//     normal number, i.e. for every quotient above ~1e-20 -- far below 0.25, the smallest quotient
//     with a non-zero e2m1 code.  Smaller quotients only decide the sign bit of a zero code, and
//     that sign is fixed up exactly (see underflow_mask8).  rb_nvfp4_selftest_division checks the
//     identity against the IEEE divide on the GPU.  Stochastic rounding, which has to match the
//     reference in distribution only, rounds q0 = RN(x*Y) itself (quot2_sr).
//   * The block-scale byte: byte(amax) = ceil_e4m3(clamp(RN(amax / 6gs))) is monotone in amax, so
//     it is e + [amax >= thr[e]], where e = RN_e4m3(amax * rup) (the hardware convert, with rup a
//     hair above 1/(6gs)) is provably the byte or the one below it, and thr[e] is the smallest
//     amax whose byte exceeds e.  The 126 thresholds are found per CTA from the exact Markstein
//     evaluation (scale_threshold); rb_nvfp4_selftest_scale checks the shortcut against it.
//   * Codes come from the hardware round-to-nearest-even convert cvt.rn.satfinite.e2m1x2.f32,
//     which rounds exactly like the reference's comparison ladder (ties to the even code).
//     Stochastic rounding uses the hardware convert cvt.rs.satfinite.e2m1x4.f32 with 16 random
//     bits per element (see sr_rbits).
//   * The Hadamard fast path: radiance's rotation is a Sylvester matrix with row signs, scaled by
//     1/4 (quantize.py:647-659).  Then y_i = 1/4 * sum_j syl(j,i) * (s_j x_j) with the same
//     left-to-right rounding, since scaling by a power of two commutes with every rounding; the
//     kernel flips the input signs while unpacking, sums with packed adds and folds the 1/4 into
//     the divisor.  Any other 16x16 matrix takes a general path (multiply then add, j = 0..15).
#include <stdio.h>

#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

namespace rb {

__device__ uint32_t g_quant_status;

constexpr int kQThreads = 256;
constexpr int kQRows = 128;
constexpr int kQStages = 3;
constexpr int kQBoxBytes = 16384;        // one 128-row x 128-byte TMA box
constexpr int kQTileBytes = 2 * kQBoxBytes;

template <bool F32IN>
struct QTile {
  static constexpr int kCols = F32IN ? 64 : 128;     // tile width in elements (two boxes)
  static constexpr int kBoxCols = F32IN ? 32 : 64;   // box width in elements
};

struct QuantArgs {
  int64_t M, K;
  const float* gs;
  const float* hadamard;
  const int64_t* seed;
  uint8_t* row_packed;
  uint8_t* row_scale;
  uint8_t* col_packed;
  uint8_t* col_scale;
  int tiles_k;
  int n_tiles;
  // Grouped mode (offs != nullptr): gs[g] is the global scale of rows [offs[g], offs[g+1]); each
  // 128-row tile takes the group of its first row.
  const int64_t* offs;
  int ngroups;
  // Fused global scale (gsync != nullptr; a cooperative launch): the kernel first reduces amax|x|
  // over the whole input (x, row stride ld_bytes), meets every other CTA at a grid barrier, and
  // writes the global scale to gs_out before quantizing with it.  gsync: four words {arrivals,
  // generation, amax[2]} -- zero before the first launch, left consistent by each.
  const void* x;
  int64_t ld_bytes;
  uint32_t* gsync;
  float* gs_out;
};

// Group of row r: the last g with offs[g] <= r (empty groups share offsets with their neighbour).
__device__ __forceinline__ int group_of_row(const int64_t* offs, int ngroups, int64_t r) {
  int lo = 0, hi = ngroups - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offs + mid) <= r) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

struct QHeader {
  uint64_t full[kQStages];
  uint64_t empty[kQStages];  // one arrive per warp when it is done with the stage's tile
  // Per e4m3 byte e: (D_e, RN(1/D_e), thr_e, 0), D_e = value(e) * gs and thr_e the smallest block
  // amax whose scale byte exceeds e (NaN: none).  16-byte entries, so both loads of pick_scale
  // are aligned.
  float4 sct[128];
  float had[256];
  uint32_t sign_word[16];
  int had_fast;
};

constexpr size_t quant_smem_bytes() { return 1024 + (size_t)kQTileBytes * kQStages + sizeof(QHeader); }

// ---------------------------------------------------------------------------------------------
// Scalar helpers
// ---------------------------------------------------------------------------------------------
// Three-input maximum (one sm_100 instruction); exact, like two fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float e4m3_value(uint32_t b) {
  const uint32_t e = b >> 3, m = b & 7u;
  if (e == 0) return __uint2float_rn(m) * 0.001953125f;  // m * 2^-9 (subnormal)
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// Smallest e4m3 byte whose value is >= s, for s in [1e-12, 448] (quantize.py:180-184): round the
// fp32 mantissa up to 3 bits in the normal range, ceil(s * 2^9) in the subnormal range.
__device__ __forceinline__ uint32_t e4m3_ceil_byte(float s) {
  const uint32_t nb = ((__float_as_uint(s) + 0xFFFFFu) >> 20) - 960u;
  const uint32_t sb = __float2uint_ru(s * 512.0f);
  return s >= 0.015625f ? nb : sb;
}

// Block-scale byte for a block amax, evaluated exactly: smallest e4m3 >= clamp(RN(amax / denom),
// 1e-12, 448).  The quotient is Markstein's (rd = RN(1/denom), nd = -denom); a quotient above 512
// saturates to 448 directly, since the corrections would overflow there.
__device__ __forceinline__ uint32_t block_scale_byte(float amax, float nd, float rd) {
  const float q0 = amax * rd;
  float q = q0;
  float r = fmaf(q, nd, amax);
  q = fmaf(r, rd, q);
  r = fmaf(q, nd, amax);
  q = fmaf(r, rd, q);
  q = (q0 > 512.0f) ? 448.0f : fminf(fmaxf(q, 1e-12f), 448.0f);
  return e4m3_ceil_byte(q);
}

// The smallest non-negative float amax with block_scale_byte(amax) >= target (1 <= target <= 126).
// The byte is monotone in amax (a composition of monotone roundings); the search starts next to
// the boundary, value(target - 1) * denom, and falls back to bisection over the bit patterns of
// the non-negative floats (which order like the floats).
__device__ float scale_threshold(uint32_t target, float nd, float rd) {
  if (target <= 1) return 0.0f;  // every block's byte is at least 1 (the 1e-12 clamp)
  uint32_t a = __float_as_uint(__fmul_rn(e4m3_value(target - 1), -nd));
  if (a > 0x7F800000u) a = 0x7F800000u;
  int steps = 0;
  if (block_scale_byte(__uint_as_float(a), nd, rd) >= target) {
    while (a > 0 && steps < 16 && block_scale_byte(__uint_as_float(a - 1), nd, rd) >= target) --a, ++steps;
  } else {
    while (steps < 16 && block_scale_byte(__uint_as_float(a), nd, rd) < target) ++a, ++steps;
  }
  if (steps < 16) return __uint_as_float(a);
  uint32_t lo = 0, hi = 0x7F800000u;  // byte(+inf) = 126 >= target
  while (lo < hi) {
    const uint32_t mid = lo + ((hi - lo) >> 1);
    if (block_scale_byte(__uint_as_float(mid), nd, rd) >= target) hi = mid;
    else lo = mid + 1;
  }
  return __uint_as_float(lo);
}

// e4m3 bytes of RN(hi) (bits 8..15) and RN(lo) (bits 0..7), saturating to 448.
__device__ __forceinline__ uint32_t e4m3x2_rn(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// Scale bytes, divisors and reciprocals of two blocks from their amaxes: e = RN_e4m3(amax * rup) is
// the exact byte or the one below it, and thr_e decides; entries e and e + 1 are read together.
// (rup >= (1 + 2^-21) / (6gs) puts amax * rup above the exact quotient s; it stays below
// s (1 + 2^-19), far short of the next e4m3 rounding boundary above ceil_e4m3(s), so RN_e4m3 lands on
// ceil_e4m3(s) or the value below.  The clamps agree: e = 0 below 1e-12 where the byte is
// 1 = e + [amax >= thr_0 = 0], and e = 126 = byte at saturation, where thr_126 is NaN.)
struct BlockScale {
  uint32_t byte;
  float d, y;
};
__device__ __forceinline__ BlockScale pick_scale(float amax, uint32_t e, uint32_t sct) {
  const uint4 t = lds128(sct + 16 * e);       // (D_e, Y_e, thr_e, 0)
  const uint2 n = lds64(sct + 16 * (e + 1));  // (D_e+1, Y_e+1)
  const bool up = amax >= __uint_as_float(t.z);
  BlockScale b;
  b.byte = e + (up ? 1u : 0u);
  b.d = __uint_as_float(up ? n.x : t.x);
  b.y = __uint_as_float(up ? n.y : t.y);
  return b;
}
__device__ __forceinline__ void scale_lookup2(float a0, float a1, float rup, uint32_t sct, BlockScale& s0,
                                              BlockScale& s1) {
  const uint32_t e = e4m3x2_rn(a1 * rup, a0 * rup);
  // e <= 126 for every finite product; the clamp keeps entry e + 1 inside the table for a NaN one.
  s0 = pick_scale(a0, min(e & 0xFFu, 126u), sct);
  s1 = pick_scale(a1, min(e >> 8, 126u), sct);
}

// max(0, |a[0]|, |a[s]|, ..., |a[15 s]|) as a depth-3 tree of three-input maxima.
__device__ __forceinline__ float amax16(const float* a, int st) {
  const float m0 = fmax3(fabsf(a[0]), fabsf(a[st]), fabsf(a[2 * st]));
  const float m1 = fmax3(fabsf(a[3 * st]), fabsf(a[4 * st]), fabsf(a[5 * st]));
  const float m2 = fmax3(fabsf(a[6 * st]), fabsf(a[7 * st]), fabsf(a[8 * st]));
  const float m3 = fmax3(fabsf(a[9 * st]), fabsf(a[10 * st]), fabsf(a[11 * st]));
  const float m4 = fmax3(fabsf(a[12 * st]), fabsf(a[13 * st]), fabsf(a[14 * st]));
  return fmax3(fmax3(m0, m1, m2), fmax3(m3, m4, fabsf(a[15 * st])), 0.0f);
}

// q = RN(x / d) for a float2, given nd = -d and y = RN(1/d) (Markstein, two corrections).  The
// first product is x * y + 0, which turns a -0 numerator into +0 (the corrections keep it there):
// the reference's code for q = -0 is 0, its sign being `q < 0`.
__device__ __forceinline__ float2 div2(float2 x, float2 nd, float2 y) {
  float2 q = __ffma2_rn(x, y, make_float2(0.0f, 0.0f));
  float2 r = __ffma2_rn(q, nd, x);
  q = __ffma2_rn(r, y, q);
  r = __ffma2_rn(q, nd, x);
  return __ffma2_rn(r, y, q);
}

// The stochastic-rounding quotient: RN(x * y) with y = RN(1/d), within 1.5 ulp of x / d (+0 for a
// -0 numerator, as above).  Stochastic rounding only has to match the reference in distribution,
// and an ulp of the quotient moves the probability of rounding up by at most 2^-22, far below the
// convert's 2^-16 resolution, so the two corrections of div2 are skipped.
__device__ __forceinline__ float2 quot2_sr(float2 x, float2 y) { return __ffma2_rn(x, y, make_float2(0.0f, 0.0f)); }

// Eight quotients -> one 32-bit word of packed e2m1 codes, e0 in the low nibble.
__device__ __forceinline__ uint32_t e2m1x8(float e0, float e1, float e2, float e3, float e4, float e5, float e6,
                                           float e7) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(e0), "f"(e1), "f"(e2), "f"(e3), "f"(e4), "f"(e5), "f"(e6), "f"(e7));
  return out;
}

// Stochastic rounding of four quotients to e2m1 by the hardware convert: element i lands in
// nibble i.  The convert rounds a magnitude up with probability floor(f * 2^16) / 2^16, f the
// fraction of the grid step above the level below (quantize.py:122-138 rounds up with probability
// f), using 16 random bits per element drawn from `rbits`: with R0 = rbits[23:16]:rbits[7:0] and
// R2 = rbits[31:24]:rbits[15:8], element 0 takes R0, element 1 the bit reversal of R0, element 2
// R2 and element 3 the bit reversal of R2, and rounds up when floor(f * 2^16) + R >= 2^16.
__device__ __forceinline__ uint32_t e2m1x4_rs(float e0, float e1, float e2, float e3, uint32_t rbits) {
  uint16_t d;
  asm("cvt.rs.satfinite.e2m1x4.f32 %0, {%1, %2, %3, %4}, %5;"
      : "=h"(d)
      : "f"(e3), "f"(e2), "f"(e1), "f"(e0), "r"(rbits));
  return d;
}

// Random bits for stochastic rounding.  A unit of 32 elements (rowblock: one row's 32-column
// group; colblock: two adjacent columns' 16-row blocks) draws from its own stream:
//   S    = mix32(lo32(unit) ^ key(hi32(unit)))   (mix32: the "lowbias32" finalizer from
//          C. Wellons' hash-prospector search, public-domain constants; a bijection with full
//          avalanche)
//   r_j  = A^j S + C_j mod 2^32 (j = 0..15; a full-period LCG with the multiplier and increment of
//          PCG's 32-bit generator), each one multiply-add from S
//   rbits of convert c (elements 4c..4c+3 of the unit) = hi16(r_2c) | hi16(r_2c+1) << 16
// so every convert draws only the upper halves of two LCG words.
__device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

// Per-launch key from the 64-bit seed (read on the device through a pointer).
__device__ __forceinline__ uint32_t sr_key(const int64_t* seed) {
  const uint64_t s = (uint64_t)(*seed);
  return mix32((uint32_t)s ^ 0x9E3779B9u) ^ mix32((uint32_t)(s >> 32) + 0x7F4A7C15u);
}

// Key for unit indices sharing the same upper 32 bits.
__device__ __forceinline__ uint32_t sr_key_hi(uint32_t key, uint64_t idx) {
  const uint32_t hi = (uint32_t)(idx >> 32);
  return hi ? key ^ mix32(hi + 0x632BE5ABu) : key;
}

constexpr uint32_t kLcgA = 747796405u, kLcgC = 2891336453u;
__host__ __device__ constexpr uint32_t lcg_mul(int j) {
  uint32_t a = 1u;
  for (int i = 0; i < j; ++i) a *= kLcgA;
  return a;
}
__host__ __device__ constexpr uint32_t lcg_add(int j) {
  uint32_t c = 0u;
  for (int i = 0; i < j; ++i) c = c * kLcgA + kLcgC;
  return c;
}
__device__ __forceinline__ uint32_t sr_unit_seed(uint64_t unit, uint32_t key) {
  return mix32((uint32_t)unit ^ sr_key_hi(key, unit));
}
__device__ __forceinline__ uint32_t sr_rbits(uint32_t s, int c) {
  return __byte_perm(s * lcg_mul(2 * c) + lcg_add(2 * c), s * lcg_mul(2 * c + 1) + lcg_add(2 * c + 1), 0x7632);
}

// A quotient that rounds to +-0 must produce nibble 0 (the reference's sign is `q < 0`, false for
// -0).  Values with |v| <= T0 = RD(Dv * 2^-150) are exactly those; they can only exist in a block
// whose divisor is large compared with the smallest non-zero input magnitude, so this runs only
// for such (rare) blocks.
__device__ __forceinline__ uint32_t underflow_mask8(const float* v, int stride, float dv) {
  const float t0 = __fmul_rd(dv * 2.98023223876953125e-8f /* 2^-25 */, 2.35098870164457501594e-38f /* 2^-125 */);
  uint32_t keep = 0xFFFFFFFFu;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (fabsf(v[e * stride]) <= t0) keep &= ~(0xFu << (4 * e));
  return keep;
}

// The same for stochastic-rounding quotients (RN(x * y), not RN(x / d)): nibble 0 where q is +-0.
__device__ __forceinline__ uint32_t zero_mask8(const float* q, int stride) {
  uint32_t keep = 0xFFFFFFFFu;
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (q[e * stride] == 0.0f) keep &= ~(0xFu << (4 * e));
  return keep;
}

__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

__device__ __forceinline__ void st_global_v2(void* p, uint32_t a, uint32_t b) {
  asm volatile("st.global.v2.b32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

struct QCtx {
  uint32_t sct;      // shared address of QHeader::sct
  uint32_t had;      // shared address of QHeader::had
  float rup;         // RN(1/(6 gs)) (1 + 2^-20)
  uint32_t key;      // stochastic rounding: rowblock-form key
  uint32_t key_col;  // colblock-form key
};

// The per-byte scale table for one global scale (threads 0..127); returns rup.
__device__ __forceinline__ float build_scale_table(float4* sct, float gs) {
  const int tid = threadIdx.x;
  const float den = __fmul_rn(6.0f, gs);
  const float rd = __frcp_rn(den);
  if (tid < 128) {
    const float d = tid < 127 ? __fmul_rn(e4m3_value(tid), gs) : 1.0f;
    const float thr = tid < 126 ? scale_threshold(tid + 1, -den, rd) : __uint_as_float(0x7FFFFFFFu);
    sct[tid] = make_float4(d, __frcp_rn(d), thr, 0.0f);
  }
  return rd * 1.00000095367431640625f;  // 1 + 2^-20
}
__device__ __forceinline__ void build_tables(QHeader* hdr, float gs, QCtx& c) { c.rup = build_scale_table(hdr->sct, gs); }

// ---------------------------------------------------------------------------------------------
// Rowblock form of a tile: thread t owns row t % 128 of box t / 128.  `rk[c]` is the shared
// address of 16-byte chunk c of that box row.
// ---------------------------------------------------------------------------------------------
template <bool F32IN, bool SR>
__device__ __forceinline__ void row_part(const uint32_t (&rk)[8], const QCtx& c, const QuantArgs& a, int64_t m0,
                                         int64_t k0, int mt, bool valid) {
  constexpr int kUnits = F32IN ? 1 : 2;  // 32-column stochastic-rounding units per thread
  const int r = threadIdx.x & 127, h = threadIdx.x >> 7;
  const int64_t col0 = k0 + (F32IN ? 32 : 64) * h;
  uint32_t w[kUnits][4];
  uint32_t sb[kUnits][2];
#pragma unroll
  for (int u = 0; u < kUnits; ++u) {
    float2 v[2][8];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if constexpr (!F32IN) {
        const uint4 c0 = lds128(rk[4 * u + 2 * i]), c1 = lds128(rk[4 * u + 2 * i + 1]);
        v[i][0] = bf16x2_to_float2(c0.x); v[i][1] = bf16x2_to_float2(c0.y);
        v[i][2] = bf16x2_to_float2(c0.z); v[i][3] = bf16x2_to_float2(c0.w);
        v[i][4] = bf16x2_to_float2(c1.x); v[i][5] = bf16x2_to_float2(c1.y);
        v[i][6] = bf16x2_to_float2(c1.z); v[i][7] = bf16x2_to_float2(c1.w);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 x = lds128(rk[4 * i + q]);
          v[i][2 * q] = make_float2(__uint_as_float(x.x), __uint_as_float(x.y));
          v[i][2 * q + 1] = make_float2(__uint_as_float(x.z), __uint_as_float(x.w));
        }
      }
    }
    BlockScale bs[2];
    scale_lookup2(amax16(&v[0][0].x, 1), amax16(&v[1][0].x, 1), c.rup, c.sct, bs[0], bs[1]);
    sb[u][0] = bs[0].byte;
    sb[u][1] = bs[1].byte;
    uint32_t seed = 0;
    if constexpr (SR) seed = sr_unit_seed((uint64_t)(m0 + r) * (uint64_t)(a.K >> 5) + (uint64_t)(col0 >> 5) + u, c.key);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float d = bs[i].d, y = bs[i].y;
      // Quotients that underflow to +-0 (possible only for large divisors) must give nibble 0.
      const float risk = F32IN ? 1.0f : 65536.0f;  // smallest |x|: 2^-149 (fp32), 2^-133 (bf16)
      const bool risky = __any_sync(0xFFFFFFFFu, d >= risk) && d >= risk;
      uint32_t keep0 = 0xFFFFFFFFu, keep1 = 0xFFFFFFFFu;
      if (!SR && risky) {
        keep0 = underflow_mask8(&v[i][0].x, 1, d);
        keep1 = underflow_mask8(&v[i][4].x, 1, d);
      }
      const float2 nd = make_float2(-d, -d), yy = make_float2(y, y);
      float2 q[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) q[e] = SR ? quot2_sr(v[i][e], yy) : div2(v[i][e], nd, yy);
      if (SR && risky) {
        keep0 = zero_mask8(&q[0].x, 1);
        keep1 = zero_mask8(&q[4].x, 1);
      }
      if constexpr (SR) {
        const uint32_t h0 = e2m1x4_rs(q[0].x, q[0].y, q[1].x, q[1].y, sr_rbits(seed, 4 * i));
        const uint32_t h1 = e2m1x4_rs(q[2].x, q[2].y, q[3].x, q[3].y, sr_rbits(seed, 4 * i + 1));
        const uint32_t h2 = e2m1x4_rs(q[4].x, q[4].y, q[5].x, q[5].y, sr_rbits(seed, 4 * i + 2));
        const uint32_t h3 = e2m1x4_rs(q[6].x, q[6].y, q[7].x, q[7].y, sr_rbits(seed, 4 * i + 3));
        w[u][2 * i] = __byte_perm(h0, h1, 0x5410);
        w[u][2 * i + 1] = __byte_perm(h2, h3, 0x5410);
      } else {
        w[u][2 * i] = e2m1x8(q[0].x, q[0].y, q[1].x, q[1].y, q[2].x, q[2].y, q[3].x, q[3].y);
        w[u][2 * i + 1] = e2m1x8(q[4].x, q[4].y, q[5].x, q[5].y, q[6].x, q[6].y, q[7].x, q[7].y);
      }
      w[u][2 * i] &= keep0;
      w[u][2 * i + 1] &= keep1;
    }
  }
  if (!valid) return;
  uint8_t* prow = a.row_packed + (m0 + r) * (a.K >> 1) + (col0 >> 1);
  st_global_v4(prow, w[0][0], w[0][1], w[0][2], w[0][3]);
  if constexpr (!F32IN) st_global_v4(prow + 16, w[1][0], w[1][1], w[1][2], w[1][3]);
  // Scale bytes: atom (mt, col0 / 64), 16-byte row r % 32, 4-byte group r / 32, byte (col0 % 64) / 16.
  uint8_t* atom = a.row_scale + ((int64_t)mt * (a.K >> 6) + (col0 >> 6)) * 512 + (r & 31) * 16 + (r >> 5) * 4;
  if constexpr (!F32IN) {
    *reinterpret_cast<uint32_t*>(atom) = sb[0][0] | (sb[0][1] << 8) | (sb[1][0] << 16) | (sb[1][1] << 24);
  } else {
    *reinterpret_cast<uint16_t*>(atom + ((col0 & 32) ? 2 : 0)) = (uint16_t)(sb[0][0] | (sb[0][1] << 8));
  }
}

// ---------------------------------------------------------------------------------------------
// The colblock form.  A unit is the 16-row group rg of two adjacent columns (pair cp of the tile):
// two blocks, worked as float2 pairs.  `bk[k]` is (the unit's base address) ^ (k << 4) and
// `box_off` a constant: row j of the unit is at bk[j % 8] + box_off + j * 128.  Returns the unit's
// packed codes (8 bytes per column) and scale bytes.  HADM: 0 no rotation, 1 the Sylvester fast
// path (`sgn[j]` = 0 or 0x80000000, the sign of row j of the matrix), 2 any other matrix.
// ---------------------------------------------------------------------------------------------
struct ColOut {
  uint32_t wx0, wx1, wy0, wy1;  // codes of column 2cp (rows 0-7, 8-15) and of column 2cp + 1
  uint32_t bx, by;              // their scale bytes
};

template <bool F32IN, int HADM, bool SR>
__device__ __forceinline__ ColOut col_unit(const uint32_t (&bk)[8], uint32_t box_off, const uint32_t (&sgn)[16],
                                           const QCtx& c, const QuantArgs& a, int64_t m0, int64_t k0, int cp,
                                           int rg) {
  // Row j of the unit as a float2 (columns 2cp, 2cp + 1), with the row sign of the fast path.
  auto load_row = [&](int j) -> float2 {
    const uint32_t addr = bk[j & 7] + box_off + j * 128;
    if constexpr (!F32IN) {
      const uint32_t w = lds32(addr);
      if constexpr (HADM == 1) {
        // Flipping the sign bit is adding 2^31: low half (w << 16) + s, high half (w & ~0xFFFF) ^ s.
        return make_float2(__uint_as_float(w * 65536u + sgn[j]), __uint_as_float((w & 0xFFFF0000u) ^ sgn[j]));
      } else {
        return bf16x2_to_float2(w);
      }
    } else {
      const uint2 w = lds64(addr);
      if constexpr (HADM == 1) return make_float2(__uint_as_float(w.x ^ sgn[j]), __uint_as_float(w.y ^ sgn[j]));
      else return make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
    }
  };
  float2 v[16];
  float fold = 1.0f;  // the rotated values are fold * y (4 on the Hadamard fast path)
  if constexpr (HADM == 2) {
    // Any matrix: y_i = sum_j R[j][i] x_j, each product rounded, then added left to right.  Row j
    // is loaded when its turn comes (a rolled loop), so only the 16 running sums stay live.
#pragma unroll 1
    for (int j = 0; j < 16; ++j) {
      const uint32_t addr = (bk[0] ^ (uint32_t)((j & 7) << 4)) + box_off + j * 128;
      float2 x;
      if constexpr (!F32IN) {
        x = bf16x2_to_float2(lds32(addr));
      } else {
        const uint2 w = lds64(addr);
        x = make_float2(__uint_as_float(w.x), __uint_as_float(w.y));
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float h = __uint_as_float(lds32(c.had + 4 * (j * 16 + i)));
        const float2 p = make_float2(__fmul_rn(h, x.x), __fmul_rn(h, x.y));
        v[i] = j == 0 ? p : make_float2(__fadd_rn(v[i].x, p.x), __fadd_rn(v[i].y, p.y));
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = load_row(j);
  }
  if constexpr (HADM == 1) {
    // y_i = sum_j syl(j, i) v_j, summed left to right.  syl(j, i) = (-1)^popc(i & j), so after
    // term j the partial sum of output i depends only on i mod w (w = the power of two above j):
    // outputs that agree there share it.  The prefixes double at j = 1, 2, 4, 8 -- 170 adds for
    // the 16 outputs instead of 240, each output's additions unchanged and in the same order.
    float2 y[16];
    const float2 pos = make_float2(1.0f, 1.0f), neg = make_float2(-1.0f, -1.0f);
    y[0] = v[0];
    int w = 1;
#pragma unroll
    for (int j = 1; j < 16; ++j) {
      const bool grow = (j & (j - 1)) == 0;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (grow && i >= w && i < 2 * w) y[i] = __ffma2_rn(v[j], (__popc(i & j) & 1) ? neg : pos, y[i - w]);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < w) y[i] = __ffma2_rn(v[j], (__popc(i & j) & 1) ? neg : pos, y[i]);
      if (grow) w *= 2;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = y[i];
    fold = 4.0f;
  }
  const float unfold = 1.0f / fold;  // exact (1 or 1/4)
  BlockScale sx, sy;
  scale_lookup2(amax16(&v[0].x, 2) * unfold, amax16(&v[0].y, 2) * unfold, c.rup, c.sct, sx, sy);
  const uint32_t bx = sx.byte, by = sy.byte;
  const float dx = sx.d * fold, dyv = sy.d * fold;
  // Quotients that underflow to +-0 (possible only for large divisors) must give nibble 0.
  // Smallest non-zero |v|: 2^-133 for bf16 inputs and sums of them, 2^-149 otherwise.
  const float risk = (F32IN || HADM == 2) ? 1.0f : 65536.0f;
  uint32_t kx0 = 0xFFFFFFFFu, kx1 = 0xFFFFFFFFu, ky0 = 0xFFFFFFFFu, ky1 = 0xFFFFFFFFu;
  const bool risky = __any_sync(0xFFFFFFFFu, dx >= risk || dyv >= risk);
  if (!SR && risky) {
    if (dx >= risk) {
      kx0 = underflow_mask8(&v[0].x, 2, dx);
      kx1 = underflow_mask8(&v[8].x, 2, dx);
    }
    if (dyv >= risk) {
      ky0 = underflow_mask8(&v[0].y, 2, dyv);
      ky1 = underflow_mask8(&v[8].y, 2, dyv);
    }
  }
  const float2 nd = make_float2(-dx, -dyv);
  const float2 yy = make_float2(sx.y * unfold, sy.y * unfold);
  float2 q[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] = SR ? quot2_sr(v[i], yy) : div2(v[i], nd, yy);
  if (SR && risky) {
    if (dx >= risk) {
      kx0 = zero_mask8(&q[0].x, 2);
      kx1 = zero_mask8(&q[8].x, 2);
    }
    if (dyv >= risk) {
      ky0 = zero_mask8(&q[0].y, 2);
      ky1 = zero_mask8(&q[8].y, 2);
    }
  }
  uint32_t wx0, wx1, wy0, wy1;
  if constexpr (SR) {
    // Unit: column pair k0/2 + cp, 16-row group m0/16 + rg; converts 0..3 take column 2cp's rows
    // 4c..4c+3, converts 4..7 column 2cp + 1's.
    const uint64_t unit = ((uint64_t)(k0 >> 1) + (uint64_t)cp) * (uint64_t)(a.M >> 4) + (uint64_t)(m0 >> 4) + rg;
    const uint32_t s = sr_unit_seed(unit, c.key_col);
    wx0 = __byte_perm(e2m1x4_rs(q[0].x, q[1].x, q[2].x, q[3].x, sr_rbits(s, 0)),
                      e2m1x4_rs(q[4].x, q[5].x, q[6].x, q[7].x, sr_rbits(s, 1)), 0x5410);
    wx1 = __byte_perm(e2m1x4_rs(q[8].x, q[9].x, q[10].x, q[11].x, sr_rbits(s, 2)),
                      e2m1x4_rs(q[12].x, q[13].x, q[14].x, q[15].x, sr_rbits(s, 3)), 0x5410);
    wy0 = __byte_perm(e2m1x4_rs(q[0].y, q[1].y, q[2].y, q[3].y, sr_rbits(s, 4)),
                      e2m1x4_rs(q[4].y, q[5].y, q[6].y, q[7].y, sr_rbits(s, 5)), 0x5410);
    wy1 = __byte_perm(e2m1x4_rs(q[8].y, q[9].y, q[10].y, q[11].y, sr_rbits(s, 6)),
                      e2m1x4_rs(q[12].y, q[13].y, q[14].y, q[15].y, sr_rbits(s, 7)), 0x5410);
  } else {
    wx0 = e2m1x8(q[0].x, q[1].x, q[2].x, q[3].x, q[4].x, q[5].x, q[6].x, q[7].x);
    wx1 = e2m1x8(q[8].x, q[9].x, q[10].x, q[11].x, q[12].x, q[13].x, q[14].x, q[15].x);
    wy0 = e2m1x8(q[0].y, q[1].y, q[2].y, q[3].y, q[4].y, q[5].y, q[6].y, q[7].y);
    wy1 = e2m1x8(q[8].y, q[9].y, q[10].y, q[11].y, q[12].y, q[13].y, q[14].y, q[15].y);
  }
  ColOut o;
  o.wx0 = wx0 & kx0;
  o.wx1 = wx1 & kx1;
  o.wy0 = wy0 & ky0;
  o.wy1 = wy1 & ky1;
  o.bx = bx;
  o.by = by;
  return o;
}

// Stores of the colblock form.  Output row kk (input column k0 + kk) holds M/2 bytes; its scale
// bytes live in SWIZZLE_32_4_4 atom (kk / 128, m / 64) at 16-byte row kk % 32, 4-byte group
// (kk % 128) / 32, byte (m / 16) % 4.  Columns past K (the zero-filled half of a K % 128 == 64 tile)
// store only their scale bytes, as zeros: the contract's padding.
__device__ __forceinline__ uint8_t* col_scale_at(const QuantArgs& a, int64_t kk, int64_t m16) {
  return a.col_scale + ((kk >> 7) * (a.M >> 6) + (m16 >> 2)) * 512 + (kk & 31) * 16 + ((kk & 127) >> 5) * 4 + (m16 & 3);
}

// bf16 tiles: warp w owns column pairs 32 (w % 2) + lane and the 32 rows 32 (w / 2) .. +31 (two
// units), so each of its two columns gets one 16-byte run and one 2-byte run of scales.
template <int HADM, bool SR>
__device__ __forceinline__ void col_part_bf16(uint32_t tile, const uint32_t (&sgn)[16], const QCtx& c,
                                              const QuantArgs& a, int64_t m0, int64_t k0, int valid_cols) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int ch = w & 1, q = w >> 1;
  const int cp = 32 * ch + lane;
  const uint32_t base = tile + ch * kQBoxBytes + 32 * q * 128 + (((lane >> 2) & 7) << 4) + ((lane & 3) << 2);
  uint32_t bk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) bk[k] = base ^ (uint32_t)(k << 4);
  const int64_t kk = k0 + 2 * cp;
  const bool valid = 2 * cp < valid_cols;
  uint8_t* px = a.col_packed + kk * (a.M >> 1) + (m0 >> 1) + 16 * q;
  const ColOut u0 = col_unit<false, HADM, SR>(bk, 0, sgn, c, a, m0, k0, cp, 2 * q);
  if constexpr (HADM == 2) {  // the general rotation: store each unit at once (fewer live registers)
    if (valid) {
      st_global_v2(px, u0.wx0, u0.wx1);
      st_global_v2(px + (a.M >> 1), u0.wy0, u0.wy1);
    }
  }
  const ColOut u1 = col_unit<false, HADM, SR>(bk, 16 * 128, sgn, c, a, m0, k0, cp, 2 * q + 1);
  if (valid) {
    if constexpr (HADM == 2) {
      st_global_v2(px + 8, u1.wx0, u1.wx1);
      st_global_v2(px + (a.M >> 1) + 8, u1.wy0, u1.wy1);
    } else {
      st_global_v4(px, u0.wx0, u0.wx1, u1.wx0, u1.wx1);
      st_global_v4(px + (a.M >> 1), u0.wy0, u0.wy1, u1.wy0, u1.wy1);
    }
  }
  const int64_t m16 = (m0 >> 4) + 2 * q;
  *reinterpret_cast<uint16_t*>(col_scale_at(a, kk, m16)) = valid ? (uint16_t)(u0.bx | (u1.bx << 8)) : (uint16_t)0;
  *reinterpret_cast<uint16_t*>(col_scale_at(a, kk + 1, m16)) = valid ? (uint16_t)(u0.by | (u1.by << 8)) : (uint16_t)0;
}

// fp32 tiles (32 column pairs): warp w owns rows 16w..16w+15 of pair `lane` (one unit).
template <int HADM, bool SR>
__device__ __forceinline__ void col_part_f32(uint32_t tile, const uint32_t (&sgn)[16], const QCtx& c,
                                             const QuantArgs& a, int64_t m0, int64_t k0) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t base = tile + (lane >> 4) * kQBoxBytes + 16 * w * 128 + (((lane & 15) >> 1) << 4) + ((lane & 1) << 3);
  uint32_t bk[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) bk[k] = base ^ (uint32_t)(k << 4);
  const ColOut u = col_unit<true, HADM, SR>(bk, 0, sgn, c, a, m0, k0, lane, w);
  const int64_t kk = k0 + 2 * lane;
  uint8_t* px = a.col_packed + kk * (a.M >> 1) + (m0 >> 1) + 8 * w;
  st_global_v2(px, u.wx0, u.wx1);
  st_global_v2(px + (a.M >> 1), u.wy0, u.wy1);
  const int64_t m16 = (m0 >> 4) + w;
  *col_scale_at(a, kk, m16) = (uint8_t)u.bx;
  *col_scale_at(a, kk + 1, m16) = (uint8_t)u.by;
  // K % 128 == 64: the last 64-column tile also zeroes the padding rows kk + 64 of its atoms.
  if ((a.K & 127) != 0 && k0 + 64 == a.K) {
    *col_scale_at(a, kk + 64, m16) = 0;
    *col_scale_at(a, kk + 65, m16) = 0;
  }
}

// ---------------------------------------------------------------------------------------------
// Fused global scale: amax over the whole input, a grid barrier, then gs for every CTA
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every thread of every CTA calls this (the launch is cooperative, so all CTAs are resident).  Each
// warp scans whole rows with 16-byte loads (rows are 16-byte aligned: the quantizer's contract),
// folding max |x| as fp32 bit patterns (non-negative floats order like their bits; NaN sorts above
// infinity and propagates, as torch's amax does).  Thread 0 of each CTA folds the CTA's maximum
// into amax[g & 1] of the generation g it read on entry and arrives at the barrier; the last to
// arrive clears the arrival count and the other amax word (the next launch's), then releases the
// generation.  Returns the global scale max(amax / 2688, 1e-12) (quantize.py:205-213), or -1 in
// every thread if the barrier wait ran out (the kernel then reports status 1 and stops).
template <bool F32IN>
__device__ float fused_global_scale(const QuantArgs& a, uint32_t* red) {
  constexpr int kPer = F32IN ? 4 : 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nvec = a.K / kPer;
  const int64_t gwarp = (int64_t)blockIdx.x * (kQThreads / 32) + warp;
  const int64_t nwarps = (int64_t)gridDim.x * (kQThreads / 32);
  uint32_t g = 0;
  if (threadIdx.x == 0) g = ld_acquire_u32(a.gsync + 1);
  uint32_t m = 0;
  for (int64_t r = gwarp; r < a.M; r += nwarps) {
    const uint4* row = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.x) + r * a.ld_bytes);
    for (int64_t c = lane; c < nvec; c += 32) {
      const uint4 v = __ldg(row + c);
      if constexpr (F32IN) {
        m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
      } else {
        m = __vmaxu2(m, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu), __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
      }
    }
  }
  if constexpr (!F32IN) m = max(m & 0xFFFFu, m >> 16) << 16;  // bf16 bits -> fp32 bits
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kQThreads / 32; ++w) m = max(m, red[w]);
    uint32_t* amax = a.gsync + 2;
    atomicMax(amax + (g & 1), m);
    __threadfence();
    bool ok = true;
    if (atomicAdd(a.gsync, 1u) == gridDim.x - 1) {
      atomicExch(a.gsync, 0u);
      atomicExch(amax + ((g + 1) & 1), 0u);
      __threadfence();
      atomicExch(a.gsync + 1, g + 1);
    } else {
      const long long start = clock64();
      while (ld_acquire_u32(a.gsync + 1) == g) {
        if (clock64() - start > kWaitLimitCycles) {
          ok = false;
          break;
        }
        __nanosleep(64);
      }
    }
    float gs = -1.0f;
    if (ok) {
      const uint32_t mb = ld_acquire_u32(amax + (g & 1));
      gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);  // amax / (6 * 448), one IEEE divide
      gs = (gs < 1e-12f) ? 1e-12f : gs;             // clamp(min=1e-12); NaN passes through
      if (blockIdx.x == 0) *a.gs_out = gs;
    }
    red[0] = __float_as_uint(gs);
  }
  __syncthreads();
  return __uint_as_float(red[0]);
}

// ---------------------------------------------------------------------------------------------
// The tile loop and the kernel
// ---------------------------------------------------------------------------------------------
template <bool F32IN>
__device__ __forceinline__ void issue_tile(const CUtensorMap& tmap, const QuantArgs& a, QHeader* hdr, uint8_t* smem,
                                           int it) {
  const int s = it % kQStages;
  const int t = (int)blockIdx.x + it * (int)gridDim.x;
  const int mt = t / a.tiles_k, kt = t - mt * a.tiles_k;
  uint8_t* dst = smem + (size_t)s * kQTileBytes;
  mbar_arrive_expect_tx(&hdr->full[s], kQTileBytes);
  tma_load_2d(dst, &tmap, &hdr->full[s], kt * QTile<F32IN>::kCols, mt * kQRows);
  tma_load_2d(dst + kQBoxBytes, &tmap, &hdr->full[s], kt * QTile<F32IN>::kCols + QTile<F32IN>::kBoxCols,
              mt * kQRows);
}

// The warps of a CTA run decoupled: each waits for a tile's TMA data on its own, works its part,
// and releases the stage with one arrive on the stage's `empty` barrier.  Warp 0 refills a stage one
// tile late -- after finishing tile it, it waits for every warp's release of tile it - 1 and loads
// tile it - 1 + S into that stage -- so no warp ever waits at a block-wide barrier for the slowest
// one (grouped launches still meet at one when a tile's group changes the scale tables).  A wait
// that runs out records its status; the warp then skips the remaining work, still arriving where
// the others count on it, with no further waiting.
template <bool F32IN, bool DO_ROW, bool DO_COL, int HADM, bool SR>
__device__ __forceinline__ void quant_loop(const CUtensorMap& tmap, const QuantArgs& a, QHeader* hdr, uint8_t* smem,
                                           QCtx& c, uint32_t cur_gs, int n_my) {
  constexpr int S = kQStages;
  constexpr int kCols = QTile<F32IN>::kCols;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t sgn[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) sgn[j] = (HADM == 1) ? hdr->sign_word[j] : 0u;
  bool failed = false;  // warp-uniform

  for (int it = 0; it < n_my; ++it) {
    const int s = it % S;
    const bool ok = __all_sync(0xFFFFFFFFu, mbar_wait(&hdr->full[s], (uint32_t)((it / S) & 1),
                                                      failed ? 0 : kWaitLimitCycles));
    if (!ok && !failed) {
      failed = true;
      if (lane == 0) record_status(&g_quant_status, kStatusTimeoutTma);
    }
    const int t = (int)blockIdx.x + it * (int)gridDim.x;
    const int mt = t / a.tiles_k, kt = t - mt * a.tiles_k;
    const int64_t m0 = (int64_t)mt * kQRows, k0 = (int64_t)kt * kCols;
    const int valid_cols = (int)min((int64_t)kCols, a.K - k0);
    if (a.offs != nullptr) {
      // A tile of another group: rebuild the tables for its global scale once every warp is done
      // with the previous tile (the condition is the same in every warp).
      const float gt = a.gs[group_of_row(a.offs, a.ngroups, m0)];
      if (__float_as_uint(gt) != cur_gs) {
        cur_gs = __float_as_uint(gt);
        __syncthreads();
        build_tables(hdr, gt, c);
        __syncthreads();
      }
    }
    if (!failed) {
      const uint32_t tile = smem_u32(smem + (size_t)s * kQTileBytes);
      if constexpr (DO_COL) {
        if constexpr (!F32IN) col_part_bf16<HADM, SR>(tile, sgn, c, a, m0, k0, valid_cols);
        else col_part_f32<HADM, SR>(tile, sgn, c, a, m0, k0);
      }
      if constexpr (DO_ROW) {
        const int r = tid & 127, h = tid >> 7;
        const uint32_t rb = tile + h * kQBoxBytes + r * 128 + ((r & 7) << 4);
        uint32_t rk[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) rk[k] = rb ^ (uint32_t)(k << 4);
        row_part<F32IN, SR>(rk, c, a, m0, k0, mt, (F32IN ? 32 : 64) * h < valid_cols);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&hdr->empty[s]);  // this warp is done reading the stage
    if (warp == 0 && it >= 1 && it - 1 + S < n_my) {
      const int ps = (it - 1) % S;
      bool e = false;
      if (lane == 0 && !failed) {
        e = mbar_wait(&hdr->empty[ps], (uint32_t)(((it - 1) / S) & 1));
        if (e) issue_tile<F32IN>(tmap, a, hdr, smem, it - 1 + S);
        else record_status(&g_quant_status, kStatusTimeoutProducer);
      }
      e = __shfl_sync(0xFFFFFFFFu, e, 0);
      if (!e) failed = true;
    }
  }
}

// The general-rotation loop as a separate (not inlined) function: it holds more values live than
// the Sylvester fast path, and keeping it out of the kernel body leaves the fast path's register
// allocation to itself.
template <bool F32IN, bool DO_ROW, bool DO_COL, bool SR>
__device__ __noinline__ void quant_loop_general(const CUtensorMap& tmap, const QuantArgs& a, QHeader* hdr,
                                                uint8_t* smem, QCtx& c, uint32_t cur_gs, int n_my) {
  quant_loop<F32IN, DO_ROW, DO_COL, 2, SR>(tmap, a, hdr, smem, c, cur_gs, n_my);
}

template <bool F32IN, bool DO_ROW, bool DO_COL, bool HAD, bool SR>
__global__ void __launch_bounds__(kQThreads, 2)
    nvfp4_quantize_kernel(const __grid_constant__ CUtensorMap tmap, const QuantArgs a) {
  constexpr int S = kQStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  QHeader* hdr = reinterpret_cast<QHeader*>(smem + (size_t)kQTileBytes * S);
  const int tid = threadIdx.x;

  if ((int)blockIdx.x >= a.n_tiles) return;
  const int n_my = (a.n_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&hdr->full[s], 1);
      mbar_init(&hdr->empty[s], kQThreads / 32);
    }
    fence_mbar_init();
    prefetch_tensormap(&tmap);
  }
  __syncthreads();
  if (tid == 0) {
    for (int it = 0; it < S && it < n_my; ++it) issue_tile<F32IN>(tmap, a, hdr, smem, it);
  }
  QCtx c;
  c.sct = smem_u32(hdr->sct);
  c.had = smem_u32(hdr->had);
  c.key = 0;
  c.key_col = 0;
  float gs;
  if (a.gsync != nullptr) {
    // The global scale of the whole input, computed here while the first tiles are in flight.
    gs = fused_global_scale<F32IN>(a, reinterpret_cast<uint32_t*>(hdr->sign_word));
    if (gs < 0.0f) {
      if (tid == 0) {
        record_status(&g_quant_status, kStatusTimeoutTma);
        for (int it = 0; it < S && it < n_my; ++it) mbar_wait(&hdr->full[it], 0);  // the copies in flight
      }
      __syncthreads();
      return;
    }
  } else {
    const int first_group =
        (a.offs != nullptr) ? group_of_row(a.offs, a.ngroups, (int64_t)((int)blockIdx.x / a.tiles_k) * kQRows) : 0;
    gs = a.gs[first_group];
  }
  build_tables(hdr, gs, c);
  if constexpr (HAD) hdr->had[tid] = a.hadamard[tid];
  if constexpr (SR) {
    c.key = sr_key(a.seed);
    c.key_col = mix32(c.key ^ 0x85EBCA6Bu);
  }
  __syncthreads();
  if constexpr (HAD) {
    // Is R = (Sylvester / 4) with row signs?  Then take the add-only fast path.
    if (tid < 32) {
      bool ok = true;
      for (int e = tid; e < 256; e += 32) {
        const int j = e >> 4, i = e & 15;
        const float rj = hdr->had[j * 16];
        const float want = (__popc(i & j) & 1) ? -rj : rj;
        ok = ok && (hdr->had[e] == want) && (fabsf(rj) == 0.25f);
      }
      ok = __all_sync(0xFFFFFFFFu, ok);
      if (tid < 16) hdr->sign_word[tid] = (hdr->had[tid * 16] < 0.0f) ? 0x80000000u : 0u;
      if (tid == 0) hdr->had_fast = ok ? 1 : 0;
    }
    __syncthreads();
    if (hdr->had_fast) quant_loop<F32IN, DO_ROW, DO_COL, 1, SR>(tmap, a, hdr, smem, c, __float_as_uint(gs), n_my);
    else quant_loop_general<F32IN, DO_ROW, DO_COL, SR>(tmap, a, hdr, smem, c, __float_as_uint(gs), n_my);
  } else {
    quant_loop<F32IN, DO_ROW, DO_COL, 0, SR>(tmap, a, hdr, smem, c, __float_as_uint(gs), n_my);
  }
}

// ---------------------------------------------------------------------------------------------
// amax -> global scale
// ---------------------------------------------------------------------------------------------
template <bool F32IN>
__global__ void __launch_bounds__(512) global_scale_kernel(const void* x, int64_t rows, int64_t cols, int64_t ld,
                                                           uint32_t* ws, float* gs_out) {
  uint32_t m = 0;  // max of |x| bit patterns (non-negative floats order like their bits)
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const bool flat = (ld == cols) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (flat) {
    const int64_t n = rows * cols;
    constexpr int kPer = F32IN ? 4 : 8;
    const int64_t nv = n / kPer;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    int64_t i = gtid;
    for (; i + 3 * stride < nv; i += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(xv + i + u * stride);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if constexpr (F32IN) {
          m = max(m, max(max(v[u].x & 0x7FFFFFFFu, v[u].y & 0x7FFFFFFFu), max(v[u].z & 0x7FFFFFFFu, v[u].w & 0x7FFFFFFFu)));
        } else {
          m = __vmaxu2(m, __vmaxu2(__vmaxu2(v[u].x & 0x7FFF7FFFu, v[u].y & 0x7FFF7FFFu),
                                   __vmaxu2(v[u].z & 0x7FFF7FFFu, v[u].w & 0x7FFF7FFFu)));
        }
      }
    }
    for (; i < nv; i += stride) {
      const uint4 v = __ldg(xv + i);
      if constexpr (F32IN) {
        m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
      } else {
        m = __vmaxu2(m, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu), __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
      }
    }
    for (int64_t e = nv * kPer + gtid; e < n; e += stride) {
      if constexpr (F32IN) m = max(m, reinterpret_cast<const uint32_t*>(x)[e] & 0x7FFFFFFFu);
      else m = max(m, (uint32_t)(reinterpret_cast<const uint16_t*>(x)[e] & 0x7FFFu));
    }
  } else if (((reinterpret_cast<uintptr_t>(x) | (uintptr_t)(ld * (F32IN ? 4 : 2)) |
               (uintptr_t)(cols * (F32IN ? 4 : 2))) & 15) == 0) {
    // Row-strided with 16-byte aligned rows (a column slice of a wider tensor): one warp per row,
    // 16-byte loads along it.
    constexpr int kPer = F32IN ? 4 : 8;
    const int lane = threadIdx.x & 31;
    const int64_t warp_id = gtid >> 5, nwarps = stride >> 5;
    const int64_t nvec = cols / kPer, ldv = ld / kPer;
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    for (int64_t r = warp_id; r < rows; r += nwarps) {
      for (int64_t c = lane; c < nvec; c += 32) {
        const uint4 v = __ldg(xv + r * ldv + c);
        if constexpr (F32IN) {
          m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
        } else {
          m = __vmaxu2(m, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu),
                                   __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
        }
      }
    }
  } else {
    for (int64_t e = gtid; e < rows * cols; e += stride) {
      const int64_t r = e / cols, c = e - r * cols;
      if constexpr (F32IN) m = max(m, reinterpret_cast<const uint32_t*>(x)[r * ld + c] & 0x7FFFFFFFu);
      else m = max(m, (uint32_t)(reinterpret_cast<const uint16_t*>(x)[r * ld + c] & 0x7FFFu));
    }
  }
  if constexpr (!F32IN) m = max(m & 0xFFFFu, m >> 16) << 16;  // bf16 bits -> fp32 bits
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t red[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      atomicMax(&ws[0], m);
      __threadfence();
      const uint32_t ticket = atomicAdd(&ws[1], 1u);
      if (ticket == gridDim.x - 1) {
        __threadfence();
        const uint32_t mb = atomicExch(&ws[0], 0u);
        atomicExch(&ws[1], 0u);
        float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);
        gs = (gs < 1e-12f) ? 1e-12f : gs;  // clamp(min=1e-12); NaN passes through as in torch
        *gs_out = gs;
      }
    }
  }
}

// Per-group global scales: group g is rows [offs[g], offs[g+1]).  Each warp scans a contiguous run
// of rows, 16 bytes per lane per load, and folds its running maximum into the group's workspace
// word whenever its run crosses into the next group; the last block to finish converts every
// group's maximum (quantize.py:205-213 per group) and resets the workspace.
template <bool F32IN>
__global__ void __launch_bounds__(256) global_scale_grouped_kernel(const void* x, int64_t rows, int64_t cols,
                                                                   int64_t ld, const int64_t* offs, int ngroups,
                                                                   uint32_t* ws, float* gs_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t limit = min(rows, __ldg(offs + ngroups));
  const int64_t per = (rows + nwarps - 1) / nwarps;
  const int64_t r0 = max(warp_id * per, __ldg(offs)), r1 = min(limit, warp_id * per + per);
  constexpr int kPer = F32IN ? 4 : 8;  // elements per 16-byte load
  const int64_t nvec = cols / kPer;
  const size_t row_bytes = (size_t)ld * (F32IN ? 4 : 2);
  int gcur = -1;
  int64_t gend = -1;
  uint32_t m = 0;
  auto flush = [&]() {
    uint32_t v = m;
    if constexpr (!F32IN) v = max(v & 0xFFFFu, v >> 16) << 16;  // bf16 bits -> fp32 bits
    v = __reduce_max_sync(0xFFFFFFFFu, v);
    if (lane == 0 && gcur >= 0) {
      atomicMax(&ws[gcur], v);
      __threadfence();
    }
    m = 0;
  };
  for (int64_t r = r0; r < r1; ++r) {
    if (r >= gend) {
      flush();
      gcur = group_of_row(offs, ngroups, r);
      gend = __ldg(offs + gcur + 1);
    }
    const uint4* row = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(x) + (size_t)r * row_bytes);
    for (int64_t c = lane; c < nvec; c += 32) {
      const uint4 v = __ldg(row + c);
      if constexpr (F32IN) {
        m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
      } else {
        m = __vmaxu2(m, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu), __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
      }
    }
  }
  flush();
  __shared__ int last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(&ws[ngroups], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last) {
    __threadfence();
    for (int gi = threadIdx.x; gi < ngroups; gi += blockDim.x) {
      const uint32_t mb = atomicExch(&ws[gi], 0u);
      float gsv = __fdiv_rn(__uint_as_float(mb), 2688.0f);
      gs_out[gi] = (gsv < 1e-12f) ? 1e-12f : gsv;
    }
    if (threadIdx.x == 0) atomicExch(&ws[ngroups], 0u);
  }
}

// Global scale and column sums in one read (the upstream gradient of a linear with a bias needs
// both: gs for its quantization and dY.sum(0) for the bias gradient, linear.py:146).  Block
// (bx, by) covers the column chunk bx (8 bf16 or 4 fp32 columns per thread, one 16-byte load per
// row) over the row range by; each thread keeps its columns' fp32 sums in registers and writes
// them to partial-sum row `by` of the workspace.  The maximum goes through ws[0] and the last
// block finalizes gs as global_scale_kernel does; colsum_finish_kernel then adds the partial rows
// in order, so the sums are deterministic.
template <bool F32IN>
__global__ void __launch_bounds__(256) global_scale_colsum_kernel(const void* x, int64_t rows, int64_t cols,
                                                                  int64_t ld, int64_t rows_per_block, uint32_t* ws,
                                                                  float* partial, float* gs_out) {
  constexpr int kPer = F32IN ? 4 : 8;
  const int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * kPer;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_block;
  const int64_t r1 = min(rows, r0 + rows_per_block);
  float acc[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) acc[e] = 0.0f;
  uint32_t m = 0;
  if (c0 < cols) {
    const size_t esize = F32IN ? 4 : 2;
    const uint8_t* base = reinterpret_cast<const uint8_t*>(x) + (size_t)c0 * esize;
    const size_t pitch = (size_t)ld * esize;
    int64_t r = r0;
    auto add = [&](const uint4 v) {
      if constexpr (F32IN) {
        acc[0] += __uint_as_float(v.x); acc[1] += __uint_as_float(v.y);
        acc[2] += __uint_as_float(v.z); acc[3] += __uint_as_float(v.w);
        m = max(m, max(max(v.x & 0x7FFFFFFFu, v.y & 0x7FFFFFFFu), max(v.z & 0x7FFFFFFFu, v.w & 0x7FFFFFFFu)));
      } else {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc[2 * q] += __uint_as_float(w[q] << 16);
          acc[2 * q + 1] += __uint_as_float(w[q] & 0xFFFF0000u);
        }
        m = __vmaxu2(m, __vmaxu2(__vmaxu2(v.x & 0x7FFF7FFFu, v.y & 0x7FFF7FFFu), __vmaxu2(v.z & 0x7FFF7FFFu, v.w & 0x7FFF7FFFu)));
      }
    };
    for (; r + 4 <= r1; r += 4) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = __ldg(reinterpret_cast<const uint4*>(base + (size_t)(r + u) * pitch));
#pragma unroll
      for (int u = 0; u < 4; ++u) add(v[u]);
    }
    for (; r < r1; ++r) add(__ldg(reinterpret_cast<const uint4*>(base + (size_t)r * pitch)));
    float* out = partial + (size_t)blockIdx.y * (size_t)cols + c0;
#pragma unroll
    for (int e = 0; e < kPer; ++e) out[e] = acc[e];
  }
  if constexpr (!F32IN) m = max(m & 0xFFFFu, m >> 16) << 16;  // bf16 bits -> fp32 bits
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      atomicMax(&ws[0], m);
      __threadfence();
      const uint32_t ticket = atomicAdd(&ws[1], 1u);
      if (ticket == gridDim.x * gridDim.y - 1) {
        __threadfence();
        const uint32_t mb = atomicExch(&ws[0], 0u);
        atomicExch(&ws[1], 0u);
        float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);
        gs = (gs < 1e-12f) ? 1e-12f : gs;
        *gs_out = gs;
      }
    }
  }
}

// colsum[c] = sum over the partial-sum rows y = 0 .. nparts-1 of partial[y][c], in that order.
__global__ void __launch_bounds__(256) colsum_finish_kernel(const float* partial, int64_t nparts, int64_t cols,
                                                            float* colsum) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float s = 0.0f;
  for (int64_t y = 0; y < nparts; ++y) s += partial[y * cols + c];
  colsum[c] = s;
}

__global__ void fill_float_kernel(float* p, float v) { *p = v; }

// Failure-path self-test: one CTA waits on an mbarrier that nothing ever arrives on (no TMA, no MMA
// is issued, so nothing is in flight when it gives up), with the tile loop's bounded wait shortened
// to `limit` cycles.  When the wait runs out the CTA records kStatusTimeoutTma in the quantizer's
// status word, exactly as the tile loop does, and returns.  `waited` receives the cycles spent.
__global__ void selftest_wait_timeout_kernel(long long limit, uint32_t* waited) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  const long long t0 = clock64();
  const bool ok = mbar_wait(&bar, 0, limit);
  const long long t1 = clock64();
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) {
      record_status(&g_quant_status, kStatusTimeoutTma);
      *waited = (uint32_t)min(t1 - t0, (long long)0xFFFFFFFF);
    }
    return;
  }
}

__global__ void selftest_division_kernel(const float* x, const float* d, int64_t n, uint32_t* mismatches) {
  uint32_t bad = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float dv = d[i];
    const float y = __frcp_rn(dv);
    const float2 q = div2(make_float2(x[i], x[i]), make_float2(-dv, -dv), make_float2(y, y));
    const float ref = __fdiv_rn(x[i], dv);
    bad += (__float_as_uint(q.x) != __float_as_uint(ref)) ? 1u : 0u;
  }
  bad = __reduce_add_sync(0xFFFFFFFFu, bad);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// Compares the scale lookup (scale_lookup2 with the per-CTA table) with the exact
// evaluation for amax[i] under the global scale *gs; counts mismatches.
__global__ void __launch_bounds__(256) selftest_scale_kernel(const float* amax, int64_t n, const float* gs,
                                                             uint32_t* mismatches) {
  __shared__ float4 sct[128];
  const float g = *gs;
  const float den = __fmul_rn(6.0f, g), rd = __frcp_rn(den);
  const float rup = build_scale_table(sct, g);
  __syncthreads();
  const uint32_t sct_addr = smem_u32(sct);
  uint32_t bad = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float a0 = amax[i];
    BlockScale s0, s1;
    scale_lookup2(a0, a0, rup, sct_addr, s0, s1);
    const uint32_t want = block_scale_byte(a0, -den, rd);
    const float d = __fmul_rn(e4m3_value(want), g);
    bad += (s0.byte != want || s0.d != d || s0.y != __frcp_rn(d)) ? 1u : 0u;
  }
  bad = __reduce_add_sync(0xFFFFFFFFu, bad);
  if ((threadIdx.x & 31) == 0 && bad) atomicAdd(mismatches, bad);
}

// The optimizer's last in-place step on a weight, w <- w + alpha * u (radiance's Muon step ends
// with target.add_(orthogonalize(u), alpha=-lr*scale), src/radiance/optim.py:518), with the global
// scale of the updated weight (quantize.py:205-213) from the same pass.  The weight's cache refresh
// can then quantize both layouts without a separate amax read.  Each element: one fp32 fused
// multiply-add of the widened operands, rounded once to w's dtype.  n elements, contiguous; ws is the
// global-scale workspace ({max bits, ticket}, zero on entry, left zero).
template <bool W_F32, bool U_F32>
__global__ void __launch_bounds__(512) update_global_scale_kernel(void* w, const void* u, int64_t n, float alpha,
                                                                  uint32_t* ws, float* gs_out) {
  uint32_t m = 0;  // max of |w'| as fp32 bit patterns
  const int64_t gtid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto load = [](const void* p, int64_t e, bool f32) -> float {
    return f32 ? reinterpret_cast<const float*>(p)[e]
               : __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p)[e] << 16);
  };
  for (int64_t e = gtid; e < n; e += stride) {
    const float r = __fmaf_rn(alpha, load(u, e, U_F32), load(w, e, W_F32));
    uint32_t rb;
    if constexpr (W_F32) {
      reinterpret_cast<float*>(w)[e] = r;
      rb = __float_as_uint(r);
    } else {
      const __nv_bfloat16 h = __float2bfloat16_rn(r);
      const uint16_t hb = *reinterpret_cast<const uint16_t*>(&h);
      reinterpret_cast<uint16_t*>(w)[e] = hb;
      rb = (uint32_t)hb << 16;
    }
    m = max(m, rb & 0x7FFFFFFFu);
  }
  m = __reduce_max_sync(0xFFFFFFFFu, m);
  __shared__ uint32_t red[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0u;
    m = __reduce_max_sync(0xFFFFFFFFu, m);
    if (lane == 0) {
      atomicMax(&ws[0], m);
      __threadfence();
      if (atomicAdd(&ws[1], 1u) == gridDim.x - 1) {
        __threadfence();
        const uint32_t mb = atomicExch(&ws[0], 0u);
        atomicExch(&ws[1], 0u);
        float gs = __fdiv_rn(__uint_as_float(mb), 2688.0f);
        gs = (gs < 1e-12f) ? 1e-12f : gs;  // clamp(min=1e-12); NaN passes through as in torch
        *gs_out = gs;
      }
    }
  }
}

}  // namespace rb

// =============================================================================================
// Host entry points
// =============================================================================================
using namespace rb;

static bool device_is_sm100() {
  static int cache[64] = {0};  // 0 unknown, 1 yes, 2 no
  const int dev = rb_host::current_device();
  if (dev < 0 || dev >= 64) return false;
  if (cache[dev] == 0) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cache[dev] = (major == 10) ? 1 : 2;
  }
  return cache[dev] == 1;
}

template <bool F32IN, bool DO_ROW, bool DO_COL, bool HAD, bool SR>
static int launch_quant(const CUtensorMap& tmap, const QuantArgs& a, cudaStream_t stream) {
  auto kern = nvfp4_quantize_kernel<F32IN, DO_ROW, DO_COL, HAD, SR>;
  constexpr size_t smem = quant_smem_bytes();
  static bool configured[64] = {false};
  const int dev = rb_host::current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
      rb_host::set_error("cudaFuncSetAttribute failed: %s", cudaGetErrorString(cudaGetLastError()));
      return RB_ERR_CUDA;
    }
    configured[dev] = true;
  }
  static int per_sm[64] = {0};
  if (dev >= 0 && dev < 64 && per_sm[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kQThreads, smem) != cudaSuccess || n < 1) n = 1;
    per_sm[dev] = n;
  }
  const int sms = rb_host::sm_budget(dev);
  const int slots = sms * ((dev >= 0 && dev < 64) ? per_sm[dev] : 1);
  const int grid = a.n_tiles < slots ? a.n_tiles : slots;
  if (a.gsync != nullptr) {
    // The fused global scale meets every CTA at a grid barrier: a cooperative launch guarantees
    // they are all resident (the grid never exceeds the occupancy-derived slot count).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kQThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, tmap, a);
  } else {
    kern<<<grid, kQThreads, smem, stream>>>(tmap, a);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 quantize launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

template <bool F32IN, bool DO_ROW, bool DO_COL>
static int dispatch_had_sr(const CUtensorMap& tmap, const QuantArgs& a, bool had, bool sr, cudaStream_t s) {
  if (had) {
    return sr ? launch_quant<F32IN, DO_ROW, DO_COL, DO_COL, true>(tmap, a, s)
              : launch_quant<F32IN, DO_ROW, DO_COL, DO_COL, false>(tmap, a, s);
  }
  return sr ? launch_quant<F32IN, DO_ROW, DO_COL, false, true>(tmap, a, s)
            : launch_quant<F32IN, DO_ROW, DO_COL, false, false>(tmap, a, s);
}

template <bool F32IN>
static int dispatch_forms(const CUtensorMap& tmap, const QuantArgs& a, bool row, bool col, bool had, bool sr,
                          cudaStream_t s) {
  if (row && col) return dispatch_had_sr<F32IN, true, true>(tmap, a, had, sr, s);
  if (row) return dispatch_had_sr<F32IN, true, false>(tmap, a, false, sr, s);
  return dispatch_had_sr<F32IN, false, true>(tmap, a, had, sr, s);
}

extern "C" {

uint32_t rb_internal_quant_status(int clear) {
  uint32_t v = 0;
  cudaDeviceSynchronize();
  cudaMemcpyFromSymbol(&v, rb::g_quant_status, sizeof(v));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(rb::g_quant_status, &z, sizeof(z));
  }
  return v;
}

int rb_nvfp4_global_scale(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                          void* workspace, void* stream) {
  if (gs_out == nullptr || workspace == nullptr || (x == nullptr && rows * cols > 0)) {
    rb_host::set_error("nvfp4 global_scale: null pointer argument");
    return RB_ERR_ARG;
  }
  if (dtype != RB_DTYPE_BF16 && dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 global_scale: unsupported dtype %d", dtype);
    return RB_ERR_ARG;
  }
  if (rows < 0 || cols < 0 || ld < cols) {
    rb_host::set_error("nvfp4 global_scale: bad shape rows=%lld cols=%lld ld=%lld", (long long)rows,
                       (long long)cols, (long long)ld);
    return RB_ERR_SHAPE;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 global_scale: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows * cols == 0) {
    rb::fill_float_kernel<<<1, 1, 0, s>>>(gs_out, 1e-12f);
  } else {
    const int sms = rb_host::sm_budget(rb_host::current_device());
    const int64_t per = (dtype == RB_DTYPE_BF16 ? 8 : 4) * 512 * 4;
    int64_t grid = (rows * cols + per - 1) / per;
    if (grid > 4 * sms) grid = 4 * sms;
    if (grid < 1) grid = 1;
    uint32_t* ws = reinterpret_cast<uint32_t*>(workspace);
    if (dtype == RB_DTYPE_BF16)
      rb::global_scale_kernel<false><<<(int)grid, 512, 0, s>>>(x, rows, cols, ld, ws, gs_out);
    else
      rb::global_scale_kernel<true><<<(int)grid, 512, 0, s>>>(x, rows, cols, ld, ws, gs_out);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 global_scale launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_nvfp4_update_global_scale(void* w, int w_dtype, const void* u, int u_dtype, int64_t n, float alpha,
                                 float* gs_out, void* workspace, void* stream) {
  if (gs_out == nullptr || workspace == nullptr || (n > 0 && (w == nullptr || u == nullptr)) || n < 0) {
    rb_host::set_error("nvfp4 update_global_scale: null pointer or negative size");
    return RB_ERR_ARG;
  }
  if ((w_dtype != RB_DTYPE_BF16 && w_dtype != RB_DTYPE_F32) || (u_dtype != RB_DTYPE_BF16 && u_dtype != RB_DTYPE_F32)) {
    rb_host::set_error("nvfp4 update_global_scale: unsupported dtypes %d, %d", w_dtype, u_dtype);
    return RB_ERR_ARG;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 update_global_scale: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 0) {
    rb::fill_float_kernel<<<1, 1, 0, s>>>(gs_out, 1e-12f);
  } else {
    const int sms = rb_host::sm_budget(rb_host::current_device());
    int64_t grid = (n + 4 * 512 - 1) / (4 * 512);
    if (grid > 8 * sms) grid = 8 * sms;
    uint32_t* ws = reinterpret_cast<uint32_t*>(workspace);
    const bool wf = w_dtype == RB_DTYPE_F32, uf = u_dtype == RB_DTYPE_F32;
    if (wf && uf) rb::update_global_scale_kernel<true, true><<<(int)grid, 512, 0, s>>>(w, u, n, alpha, ws, gs_out);
    else if (wf) rb::update_global_scale_kernel<true, false><<<(int)grid, 512, 0, s>>>(w, u, n, alpha, ws, gs_out);
    else if (uf) rb::update_global_scale_kernel<false, true><<<(int)grid, 512, 0, s>>>(w, u, n, alpha, ws, gs_out);
    else rb::update_global_scale_kernel<false, false><<<(int)grid, 512, 0, s>>>(w, u, n, alpha, ws, gs_out);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 update_global_scale launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

static int quantize_impl(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* gs,
                         const int64_t* offs, int ngroups, const float* hadamard, const int64_t* seed,
                         void* row_packed, void* row_scale, void* col_packed, void* col_scale, void* stream,
                         float* gs_out = nullptr, uint32_t* gsync = nullptr) {
  const bool row = row_packed != nullptr || row_scale != nullptr;
  const bool col = col_packed != nullptr || col_scale != nullptr;
  if (!row && !col) {
    rb_host::set_error("nvfp4 quantize: no output form requested");
    return RB_ERR_ARG;
  }
  if ((row && (row_packed == nullptr || row_scale == nullptr)) ||
      (col && (col_packed == nullptr || col_scale == nullptr)) || x == nullptr || gs == nullptr) {
    rb_host::set_error("nvfp4 quantize: null pointer argument");
    return RB_ERR_ARG;
  }
  if (dtype != RB_DTYPE_BF16 && dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 quantize: unsupported dtype %d", dtype);
    return RB_ERR_ARG;
  }
  if (rows <= 0 || cols <= 0 || rows % 128 != 0 || cols % 64 != 0) {
    rb_host::set_error("nvfp4 quantize needs rows %% 128 == 0 and cols %% 64 == 0, got (%lld, %lld)",
                       (long long)rows, (long long)cols);
    return RB_ERR_SHAPE;
  }
  const int esize = dtype == RB_DTYPE_BF16 ? 2 : 4;
  if (ld < cols || ((uint64_t)ld * esize) % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
    rb_host::set_error("nvfp4 quantize: input must be 16-byte aligned with a 16-byte row stride (ld=%lld)",
                       (long long)ld);
    return RB_ERR_ARG;
  }
  if ((row && ((reinterpret_cast<uintptr_t>(row_packed) & 15) || (reinterpret_cast<uintptr_t>(row_scale) & 3))) ||
      (col && (reinterpret_cast<uintptr_t>(col_packed) & 15 || (reinterpret_cast<uintptr_t>(col_scale) & 15)))) {
    rb_host::set_error("nvfp4 quantize: packed outputs must be 16-byte aligned, scales 16 (colblock) or 4 (rowblock)");
    return RB_ERR_ARG;
  }
  if ((rows / 128) * (cols / 64) > (int64_t)0x7FFFFFFF) {
    rb_host::set_error("nvfp4 quantize: tensor too large");
    return RB_ERR_SHAPE;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 quantize: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  CUtensorMap tmap;
  const bool f32 = dtype == RB_DTYPE_F32;
  if (!rb_host::make_tmap_2d(&tmap, x, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                             (uint64_t)cols, (uint64_t)rows, (uint64_t)ld * esize, f32 ? 32 : 64, 128,
                             CU_TENSOR_MAP_SWIZZLE_128B))
    return RB_ERR_CUDA;
  QuantArgs a;
  a.M = rows;
  a.K = cols;
  a.gs = gs;
  a.hadamard = hadamard;
  a.seed = seed;
  a.row_packed = reinterpret_cast<uint8_t*>(row_packed);
  a.row_scale = reinterpret_cast<uint8_t*>(row_scale);
  a.col_packed = reinterpret_cast<uint8_t*>(col_packed);
  a.col_scale = reinterpret_cast<uint8_t*>(col_scale);
  const int tile_cols = f32 ? QTile<true>::kCols : QTile<false>::kCols;
  a.tiles_k = (int)((cols + tile_cols - 1) / tile_cols);
  a.n_tiles = (int)((rows / 128) * a.tiles_k);
  a.offs = offs;
  a.ngroups = ngroups;
  a.x = x;
  a.ld_bytes = ld * esize;
  a.gsync = gsync;
  a.gs_out = gs_out;
  const bool had = col && hadamard != nullptr;
  const bool sr = seed != nullptr;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return f32 ? dispatch_forms<true>(tmap, a, row, col, had, sr, s) : dispatch_forms<false>(tmap, a, row, col, had, sr, s);
}

int rb_nvfp4_quantize(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* gs,
                      const float* hadamard, const int64_t* seed, void* row_packed, void* row_scale,
                      void* col_packed, void* col_scale, void* stream) {
  return quantize_impl(x, dtype, rows, cols, ld, gs, nullptr, 0, hadamard, seed, row_packed, row_scale, col_packed,
                       col_scale, stream);
}

int rb_nvfp4_quantize_auto_scale(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                                 const float* hadamard, const int64_t* seed, void* row_packed, void* row_scale,
                                 void* col_packed, void* col_scale, void* workspace, void* stream) {
  if (gs_out == nullptr || workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 15) != 0) {
    rb_host::set_error("nvfp4 quantize_auto_scale: needs a global-scale output and a 16-byte aligned workspace");
    return RB_ERR_ARG;
  }
  return quantize_impl(x, dtype, rows, cols, ld, gs_out, nullptr, 0, hadamard, seed, row_packed, row_scale,
                       col_packed, col_scale, stream, gs_out, reinterpret_cast<uint32_t*>(workspace));
}

int rb_nvfp4_quantize_grouped(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                              const int64_t* offsets, int num_groups, const float* group_gs, const float* hadamard,
                              const int64_t* seed, void* row_packed, void* row_scale, void* col_packed,
                              void* col_scale, void* stream) {
  if (offsets == nullptr || num_groups < 1 || (reinterpret_cast<uintptr_t>(offsets) & 7) != 0) {
    rb_host::set_error("nvfp4 quantize_grouped: needs at least one group and an 8-byte aligned offsets array");
    return RB_ERR_ARG;
  }
  return quantize_impl(x, dtype, rows, cols, ld, group_gs, offsets, num_groups, hadamard, seed, row_packed,
                       row_scale, col_packed, col_scale, stream);
}

// Row splits of global_scale_colsum_kernel for a launch of `gx` column chunks: enough blocks to
// fill the GPU four times over, and at most one per row.
static int64_t colsum_parts(int64_t rows, int64_t gx) {
  const int64_t want = (4 * (int64_t)rb_host::sm_budget(rb_host::current_device()) + gx - 1) / gx;
  return max((int64_t)1, min(rows, want));
}

size_t rb_nvfp4_global_scale_colsum_workspace(int dtype, int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 16;
  const int64_t per_block = (dtype == RB_DTYPE_F32 ? 4 : 8) * 256;
  const int64_t gx = (cols + per_block - 1) / per_block;
  return 16 + (size_t)colsum_parts(rows, gx) * (size_t)cols * sizeof(float);
}

int rb_nvfp4_global_scale_colsum(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                                 float* colsum_out, void* workspace, void* stream) {
  if (x == nullptr || gs_out == nullptr || colsum_out == nullptr || workspace == nullptr) {
    rb_host::set_error("nvfp4 global_scale_colsum: null pointer argument");
    return RB_ERR_ARG;
  }
  if (dtype != RB_DTYPE_BF16 && dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 global_scale_colsum: unsupported dtype %d", dtype);
    return RB_ERR_ARG;
  }
  const int esize = dtype == RB_DTYPE_BF16 ? 2 : 4;
  if (rows <= 0 || cols <= 0 || ld < cols || (cols * esize) % 16 != 0 || ((uint64_t)ld * esize) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0 || (reinterpret_cast<uintptr_t>(workspace) & 15) != 0) {
    rb_host::set_error("nvfp4 global_scale_colsum: needs 16-byte aligned rows of a multiple of 16 bytes and a "
                       "16-byte aligned workspace (rows=%lld cols=%lld ld=%lld)", (long long)rows, (long long)cols,
                       (long long)ld);
    return RB_ERR_SHAPE;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 global_scale_colsum: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t per_block = (int64_t)(16 / esize) * 256;
  const int64_t gx = (cols + per_block - 1) / per_block;
  const int64_t parts = colsum_parts(rows, gx);
  if (gx > 0x7FFFFFFF || parts > 65535) {
    rb_host::set_error("nvfp4 global_scale_colsum: tensor too large");
    return RB_ERR_SHAPE;
  }
  const int64_t rows_per_block = (rows + parts - 1) / parts;
  const int64_t used = (rows + rows_per_block - 1) / rows_per_block;  // partial rows actually written
  uint32_t* ws = reinterpret_cast<uint32_t*>(workspace);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + 16);
  const dim3 grid((unsigned)gx, (unsigned)used);
  if (dtype == RB_DTYPE_BF16)
    rb::global_scale_colsum_kernel<false><<<grid, 256, 0, s>>>(x, rows, cols, ld, rows_per_block, ws, partial, gs_out);
  else
    rb::global_scale_colsum_kernel<true><<<grid, 256, 0, s>>>(x, rows, cols, ld, rows_per_block, ws, partial, gs_out);
  rb::colsum_finish_kernel<<<(unsigned)((cols + 255) / 256), 256, 0, s>>>(partial, used, cols, colsum_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 global_scale_colsum launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_nvfp4_global_scale_grouped(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                  const int64_t* offsets, int num_groups, float* gs_out, void* workspace,
                                  void* stream) {
  if (gs_out == nullptr || workspace == nullptr || offsets == nullptr || x == nullptr || num_groups < 1 ||
      (reinterpret_cast<uintptr_t>(offsets) & 7) != 0) {
    rb_host::set_error("nvfp4 global_scale_grouped: null pointer argument or no groups");
    return RB_ERR_ARG;
  }
  if (dtype != RB_DTYPE_BF16 && dtype != RB_DTYPE_F32) {
    rb_host::set_error("nvfp4 global_scale_grouped: unsupported dtype %d", dtype);
    return RB_ERR_ARG;
  }
  const int esize = dtype == RB_DTYPE_BF16 ? 2 : 4;
  if (rows <= 0 || cols <= 0 || ld < cols || (cols * esize) % 16 != 0 || ((uint64_t)ld * esize) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) != 0) {
    rb_host::set_error("nvfp4 global_scale_grouped: needs 16-byte aligned rows of a multiple of 16 bytes "
                       "(rows=%lld cols=%lld ld=%lld)", (long long)rows, (long long)cols, (long long)ld);
    return RB_ERR_SHAPE;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 global_scale_grouped: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int sms = rb_host::sm_budget(rb_host::current_device());
  const int64_t per = (int64_t)(16 / esize) * 256 * 8;  // ~8 loads per thread
  int64_t grid = (rows * cols + per - 1) / per;
  if (grid > 4 * sms) grid = 4 * sms;
  if (grid < 1) grid = 1;
  uint32_t* ws = reinterpret_cast<uint32_t*>(workspace);
  if (dtype == RB_DTYPE_BF16)
    rb::global_scale_grouped_kernel<false><<<(int)grid, 256, 0, s>>>(x, rows, cols, ld, offsets, num_groups, ws, gs_out);
  else
    rb::global_scale_grouped_kernel<true><<<(int)grid, 256, 0, s>>>(x, rows, cols, ld, offsets, num_groups, ws, gs_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("nvfp4 global_scale_grouped launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_nvfp4_selftest_division(const float* x, const float* d, int64_t n, uint32_t* mismatches, void* stream) {
  if (x == nullptr || d == nullptr || mismatches == nullptr || n < 0) {
    rb_host::set_error("nvfp4 selftest_division: bad arguments");
    return RB_ERR_ARG;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 selftest_division: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  const int sms = rb_host::sm_budget(rb_host::current_device());
  rb::selftest_division_kernel<<<4 * sms, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, d, n, mismatches);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("selftest launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

uint32_t rb_internal_gemm_selftest_wait(long long limit, uint32_t* waited, cudaStream_t stream);

int rb_nvfp4_selftest_wait_timeout(int which, long long limit_cycles, uint32_t* waited_cycles, void* stream) {
  if (waited_cycles == nullptr || limit_cycles <= 0 || limit_cycles > rb::kWaitLimitCycles || (which != 0 && which != 1)) {
    rb_host::set_error("nvfp4 selftest_wait_timeout: which must be 0 or 1, 0 < limit_cycles <= %lld, and "
                       "waited_cycles a device pointer", (long long)rb::kWaitLimitCycles);
    return RB_ERR_ARG;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 selftest_wait_timeout: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (which == 0) rb::selftest_wait_timeout_kernel<<<1, 128, 0, s>>>(limit_cycles, waited_cycles);
  else rb_internal_gemm_selftest_wait(limit_cycles, waited_cycles, s);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("selftest launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_nvfp4_selftest_scale(const float* amax, int64_t n, const float* gs, uint32_t* mismatches, void* stream) {
  if (amax == nullptr || gs == nullptr || mismatches == nullptr || n < 0) {
    rb_host::set_error("nvfp4 selftest_scale: bad arguments");
    return RB_ERR_ARG;
  }
  if (!device_is_sm100()) {
    rb_host::set_error("nvfp4 selftest_scale: the current device is not an sm_100 GPU");
    return RB_ERR_DEVICE;
  }
  const int sms = rb_host::sm_budget(rb_host::current_device());
  rb::selftest_scale_kernel<<<2 * sms, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(amax, n, gs, mismatches);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    rb_host::set_error("selftest launch failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // extern "C"
