/*
 * radiance_nvfp4 -- C ABI of the B200-native NVFP4 linear-layer path.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer the caller owns
 * (allocated by any allocator), every call is asynchronous on the caller's CUDA stream
 * (`stream` is a cudaStream_t, NULL for the legacy default stream), and no call synchronises the
 * host.  Global scales, the stochastic-rounding seed and the GEMM's alpha are read on the device
 * through pointers, so a sequence of calls can be captured in a CUDA graph.
 *
 * Return value: 0 on success, otherwise an RB_ERR_* code with a message available from
 * rb_nvfp4_last_error() (thread-local).  Kernels never trap: a device-side wait that runs out
 * records a code readable with rb_nvfp4_device_status().
 *
 * Layouts (identical to radiance's; src/radiance/nvfp4/quantize.py in jamespa16/radiance):
 *   packed  : uint8, two e2m1 codes per byte, element 2i in the low nibble (quantize.py:142-149).
 *   scale   : uint8 e4m3 block scales, one per 16 elements along the contraction dimension, in
 *             the flat SWIZZLE_32_4_4 order of quantize.py:271-305: scale (r, c) lives at byte
 *             ((r/128)*ceil(cols/4) + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4, zero-padded
 *             to whole 128x4 tiles.
 *   rowblock: (rows, cols) -> packed (rows, cols/2), scale tiles (rows/128) x (cols/64).
 *   colblock: (rows, cols) -> packed (cols, rows/2), scale tiles ceil(cols/128) x (rows/64)
 *             (blocks run along dim 0 and the output is transposed; quantize.py:235-268).
 */
#ifndef RADIANCE_NVFP4_H_
#define RADIANCE_NVFP4_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RB_NVFP4_ABI_VERSION 7

/* Input element types. */
#define RB_DTYPE_BF16 0
#define RB_DTYPE_F32 1

/* Output element types of the GEMMs. */
#define RB_OUT_BF16 0
#define RB_OUT_F32 1

/* Return codes. */
#define RB_OK 0
#define RB_ERR_SHAPE 1   /* a shape violates the contract (message names it, e.g. "rows % 128") */
#define RB_ERR_ARG 2     /* bad pointer, alignment, dtype or flag */
#define RB_ERR_CUDA 3    /* a CUDA runtime/driver call failed */
#define RB_ERR_DEVICE 4  /* the current device is not an sm_100 (B200-class) GPU */

/* Message for the last failing call on this thread. */
const char* rb_nvfp4_last_error(void);

/* RB_NVFP4_ABI_VERSION of the loaded library. */
int rb_nvfp4_abi_version(void);

/*
 * SM budget of this library's kernels on the current device: their grids are sized for `sms`
 * streaming multiprocessors (0 = all of them), so that kernels of another stream -- a gradient
 * reduce-scatter overlapping the backward pass -- find SMs free while ours run.  Returns the previous
 * budget.  Host-side setting for the launches that follow; no counterpart in the reference.
 */
int rb_nvfp4_set_sm_budget(int sms);

/*
 * First non-zero status recorded by any kernel of this library on the current device since the
 * last clear; 0 if none.  Synchronises the device.  Codes: 1-4 a bounded device-side wait ran out
 * (TMA data, MMA completion, accumulator hand-off, free pipeline stage); 5 a grouped-GEMM record
 * broke its contract; 6 the GEMM's whole-TMEM allocation did not start at address 0.
 * Test and debugging aid; no counterpart in the reference.
 */
int rb_nvfp4_device_status(int clear);

/*
 * Per-tensor global scale: *gs_out = max(amax(|x|) / (6 * 448), 1e-12) as fp32, one IEEE divide.
 * Replaces `global_scale_of` (quantize.py:205-213).
 *   x         : rows x cols elements of `dtype`, row stride `ld` elements (ld >= cols).
 *   workspace : 8 bytes of device memory, zero before the first call; every call leaves it zero
 *               again.  Calls that share a workspace must be ordered (same stream).
 */
int rb_nvfp4_global_scale(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                          void* workspace, void* stream);

/*
 * The same global scale as rb_nvfp4_global_scale, for callers that cannot allocate device memory
 * on the call path -- code that runs where device allocation is not allowed (a host callback),
 * plugin hosts whose execute step only receives pre-planned buffers, or a plain C/FFI caller that
 * has device pointers but no allocator.  It takes no workspace and allocates nothing; the caller
 * passes only the input and the output.  No counterpart in the reference (radiance's
 * global_scale_of allocates through torch).
 *   Scratch: a fixed 64 KiB device array inside this library (held by every GPU that loads it
 *   until exit), shared by all calls on a device.  One call covers at most 2^31 elements
 *   (rows * cols); larger inputs return RB_ERR_SHAPE.  Calls whose kernels overlap on the GPU race
 *   on the scratch: order them (for example, issue them on one stream).
 *   The first call on each device looks up the scratch's device address; make that first call
 *   before any stream capture.
 *   The call uses the scratch of the current device: x and stream must belong to it.  An x on
 *   another device returns RB_ERR_ARG.
 */
int rb_nvfp4_global_scale_noalloc(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                                  void* stream);

/*
 * NVFP4 quantizer: one pass over x writes the rowblock form, the colblock form, or both.
 * Replaces `quantize` (quantize.py:672-736) and its two Triton kernels (quantize.py:538-644);
 * bit-identical to `quantize_reference` / `ref_quantize_rowblock` / `ref_quantize_colblock`
 * (quantize.py:216-268, :412-433) on codes and scale bytes for round-to-nearest.
 *   x          : rows x cols of `dtype`, row stride ld elements; rows % 128 == 0, cols % 64 == 0,
 *                16-byte aligned base and ld*elemsize % 16 == 0.
 *   gs         : device fp32 global scale (the quantizer divides by 6*gs once per block).
 *   hadamard   : NULL or a device 16x16 fp32 matrix R; the colblock form quantizes R^T applied to
 *                every 16-row group (quantize.py:261-262).  Not applied to the rowblock form.
 *   seed       : device int64 seed for stochastic rounding (read on the device); NULL = round to
 *                nearest even.  With a seed both forms use stochastic rounding with the rule of
 *                quantize.py:122-138 (up with probability (a - lo) / (hi - lo)), resolved to
 *                2^-16 of a grid step by the hardware convert cvt.rs.satfinite.e2m1x4.f32 (up with
 *                probability floor(f * 2^16) / 2^16 for the fraction f of q = RN(x * RN(1/D)),
 *                the quotient within 1.5 ulp of x / D).  Each 32-element unit
 *                (rowblock: 32 columns of a row; colblock: a column pair's 16-row blocks) draws
 *                from its own counter-based stream keyed by the seed and the unit's index, so
 *                results depend on (seed, element position) only -- not on the launch shape --
 *                and differ from radiance's tl.rand draws.
 *   row_packed : NULL or rows x cols/2 bytes, 16-byte aligned;  row_scale: NULL or
 *                (rows/128)*(cols/64)*512 bytes, 4-byte aligned.
 *   col_packed : NULL or cols x rows/2 bytes, 16-byte aligned;  col_scale: NULL or
 *                ceil(cols/128)*(rows/64)*512 bytes, 16-byte aligned (padding rows are written as
 *                zero).
 * At least one of the two forms must be requested; each form needs both of its pointers.
 */
int rb_nvfp4_quantize(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* gs,
                      const float* hadamard, const int64_t* seed, void* row_packed, void* row_scale,
                      void* col_packed, void* col_scale, void* stream);

/*
 * rb_nvfp4_global_scale followed by rb_nvfp4_quantize, in one launch: the kernel reduces amax|x|
 * over the whole input, meets all its CTAs at a grid barrier (a cooperative launch), writes
 * *gs_out = max(amax / 2688, 1e-12) exactly as rb_nvfp4_global_scale does, and quantizes with it --
 * the same bytes as the two calls, one launch fewer, and the quantizing pass re-reads the input from
 * L2 when it fits there.  Replaces the `global_scale_of(x)` + `quantize(x, ...)` pairs of
 * linear.py:79-80 and :127-136.
 *   gs_out    : device fp32, written by the call.
 *   workspace : 16 bytes of device memory, 16-byte aligned, zeroed before the first call; every call
 *               leaves it ready for the next.  Calls that share a workspace must be ordered (same
 *               stream).
 * Other arguments, contract and outputs as rb_nvfp4_quantize.
 */
int rb_nvfp4_quantize_auto_scale(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                                 const float* hadamard, const int64_t* seed, void* row_packed, void* row_scale,
                                 void* col_packed, void* col_scale, void* workspace, void* stream);

/*
 * Block-scaled NVFP4 GEMM on the tcgen05 tensor cores:
 *   out[i, j] = (alpha_a * alpha_b) * sum_k deq(a)[i, k] * deq(b)[j, k]  (+ bias[j])
 * with deq() the e2m1 codes times their e4m3 block scales.  Replaces `nvfp4_mm` + `mm`
 * (quantize.py:359-409: torch._scaled_mm_v2 followed by the global-scale multiply and cast) and
 * the bias add of linear.py:82-83, fused into one kernel.
 *   a_packed/a_scale : rowblock-layout operand, m rows, k contraction (a "rows x contraction"
 *                      NVFP4Tensor, quantize.py:328-356).  b_packed/b_scale: likewise, n rows.
 *   alpha_a, alpha_b : device fp32 global scales of the two operands (NULL = 1).
 *   bias             : NULL or n elements of `bias_dtype` (RB_DTYPE_BF16 / RB_DTYPE_F32), 16-byte
 *                      aligned.
 *   out              : m x n of `out_dtype`, row stride ldo elements.
 *   m % 128 == 0, n % 128 == 0, k % 64 == 0.
 */
int rb_nvfp4_gemm(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale, int64_t m,
                  int64_t n, int64_t k, const float* alpha_a, const float* alpha_b, const void* bias, int bias_dtype,
                  void* out, int out_dtype, int64_t ldo, void* stream);

/*
 * rb_nvfp4_gemm whose epilogue also writes every output tile into `npeers` other GPUs' copies of
 * the output: the all-gather of an N-split layer fused into the GEMM.  Rank r of g computes
 * columns r*n .. r*n+n-1 of a (m, g*n) output and stores them into all g copies over NVLink while
 * later tiles are still being multiplied.  peer_out is a host array of npeers (<= 7) device
 * pointers, each at the position `out` has in that GPU's buffer (same ldo); the memory must be
 * mapped into this process (rb_peer_open, or peer access between the devices).  The call only writes; the caller
 * synchronises the GPUs before reading the peers' copies.  It stands in for the bf16 output
 * all-gather of the N-split layers (no reference counterpart: radiance has no N-split path).
 */
int rb_nvfp4_gemm_allgather(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale,
                            int64_t m, int64_t n, int64_t k, const float* alpha_a, const float* alpha_b,
                            const void* bias, int bias_dtype, void* out, int out_dtype, int64_t ldo,
                            void* const* peer_out, int npeers, void* stream);

/*
 * Peer buffers for rb_nvfp4_gemm_allgather, shared between the processes of one box by CUDA IPC
 * (no NVLink multicast object is created; peers touch a mapping only with plain loads and stores).
 * No reference counterpart: radiance has no multi-GPU path.
 *   rb_peer_alloc  : one cudaMalloc allocation of `bytes` (IPC needs a whole allocation).
 *   rb_peer_handle : its RB_PEER_HANDLE_BYTES-byte IPC handle, for the caller to send to the peers.
 *   rb_peer_open   : map a peer's handle into this process (peer access enabled lazily);
 *                    rb_peer_close unmaps it.  rb_peer_free frees an rb_peer_alloc allocation.
 * These synchronise like the CUDA calls they wrap; none of them may run during stream capture.
 */
#define RB_PEER_HANDLE_BYTES 64
int rb_peer_alloc(size_t bytes, void** ptr_out);
int rb_peer_free(void* ptr);
int rb_peer_handle(void* ptr, void* handle_out);
int rb_peer_open(const void* handle, void** ptr_out);
int rb_peer_close(void* ptr);

/*
 * The optimizer's last in-place step on a weight fused with the start of its cache refresh:
 * w <- w + alpha * u elementwise (radiance's Muon step ends with target.add_(orthogonalize(u),
 * alpha=-lr*scale), src/radiance/optim.py:518, and linear.py:193-210 then re-quantizes the weight),
 * and *gs_out = the updated weight's global scale as rb_nvfp4_global_scale computes it.  Each element
 * is one fp32 fused multiply-add of the widened operands, rounded once to w's dtype.
 *   w, u      : n contiguous elements each of w_dtype / u_dtype (RB_DTYPE_BF16 or RB_DTYPE_F32);
 *               w is updated in place.
 *   workspace : the 8-byte workspace of rb_nvfp4_global_scale (zeroed before the first call, left
 *               zeroed; calls ordered on one stream can share it).
 */
int rb_nvfp4_update_global_scale(void* w, int w_dtype, const void* u, int u_dtype, int64_t n, float alpha,
                                 float* gs_out, void* workspace, void* stream);

/*
 * rb_nvfp4_gemm for a SwiGLU producer (bf16 output): the gate/up projection of radiance's
 * FeedForward, h = F.silu(gate_proj(x)) * up_proj(x) (src/radiance/model/ffn.py:32), with the
 * activation and the global scale of h -- the next linear's quantizer input -- computed in the
 * epilogue, so neither h's elementwise pass nor its amax pass reads the output again.
 *   b_packed/b_scale : the gate and up weights as one n-row operand whose rows come in blocks of
 *                      64: [32 gate rows | the 32 up rows of the same hidden units]; bias (if any)
 *                      interleaved the same way.  out (m x n, bf16, row stride ldo) holds the
 *                      pre-activations in that order (kept for the SwiGLU backward).
 *   h                : m x n/2 bf16, row stride ldh elements (16-byte aligned, ldh*2 % 16 == 0):
 *                      h[i, 32c + j] = bf16(bf16(silu(g)) * u) for g = out[i, 64c + j],
 *                      u = out[i, 64c + 32 + j], silu(g) = g / (1 + exp(-g)) in fp32 -- the
 *                      roundings of the bf16 eager F.silu(g) * u.
 *   workspace        : 8 bytes, 8-byte aligned, zeroed before the first call (every call leaves it
 *                      zeroed again; calls ordered on one stream can share it).
 *   h_global_scale   : device fp32, set to max(amax|h| / 2688, 1e-12) as rb_nvfp4_global_scale
 *                      would compute it from h (quantize.py:205-213).
 *   m % 128 == 0, n % 128 == 0, k % 64 == 0 as rb_nvfp4_gemm.
 */
int rb_nvfp4_gemm_swiglu(const void* a_packed, const void* a_scale, const void* b_packed, const void* b_scale,
                         int64_t m, int64_t n, int64_t k, const float* alpha_a, const float* alpha_b, const void* bias,
                         int bias_dtype, void* out, int64_t ldo, void* h, int64_t ldh, void* workspace,
                         float* h_global_scale, void* stream);

/*
 * The backward of the SwiGLU producer (h = F.silu(g) * u, src/radiance/model/ffn.py:32) in one pass:
 *   grad_gu[r, 64c + j]      = bf16(silu_backward(bf16(grad_h * u), g))   (the gate half)
 *   grad_gu[r, 64c + 32 + j] = bf16(grad_h * bf16(silu(g)))               (the up half)
 * for g = gu[r, 64c + j], u = gu[r, 64c + 32 + j], grad_h = grad_h[r, 32c + j] -- the interleaved
 * layout of rb_nvfp4_gemm_swiglu -- with the roundings of the eager torch ops autograd runs for that
 * line (silu(g) = g / (1 + exp(-g)), silu_backward(dy, g) = dy * s * (1 + g * (1 - s)),
 * s = 1 / (1 + exp(-g)), each evaluated in fp32 from bf16 inputs and rounded to bf16), and
 * *gs_out = the global scale of grad_gu (quantize.py:205-213), the gate/up linear's next input.
 *   grad_h : rows x hidden bf16, row stride ldgh;  gu, grad_gu: rows x 2*hidden bf16, strides ldgu,
 *            ldgg.  hidden % 32 == 0, 16-byte aligned tensors, strides multiples of 8 elements.
 *   workspace : the 8-byte workspace of rb_nvfp4_global_scale.
 */
int rb_nvfp4_swiglu_backward(const void* grad_h, int64_t ldgh, const void* gu, int64_t ldgu, int64_t rows,
                             int64_t hidden, void* grad_gu, int64_t ldgg, float* gs_out, void* workspace,
                             void* stream);

/*
 * SwiGLU on pre-activations in any layout of 32-unit groups (no reference counterpart as an entry
 * point; it replaces the eager F.silu(g) * u of radiance's expert FFN, src/radiance/model/ffn.py:148-153,
 * and its autograd backward).  The gate value of (row r, hidden unit j) is
 * gate[r * ld + (j / 32) * blk + j % 32] and the up value sits at the same offset from `up`:
 *   radiance's split [gate | up] halves: up = gate + hidden, blk = 32;
 *   the interleaved order of rb_nvfp4_gemm_swiglu: up = gate + 32, blk = 64.
 * forward:  h[r, j] = bf16(bf16(silu(g)) * u), *gs_out = the global scale of h.
 * backward: grad_gate / grad_up (same scheme with blko, ldo) as rb_nvfp4_swiglu_backward computes
 *           them, *gs_out = the global scale of the whole gradient.
 * Roundings are those of the eager torch ops.  hidden % 32 == 0; bf16 tensors 16-byte aligned;
 * strides, blk and the up offsets multiples of 8 elements, up at or above gate; workspace: the
 * 8-byte workspace of rb_nvfp4_global_scale (zero on entry, left zero).
 */
int rb_nvfp4_swiglu_forward_strided(const void* gate, const void* up, int64_t ld, int64_t blk, int64_t rows,
                                    int64_t hidden, void* h, int64_t ldh, float* gs_out, void* workspace,
                                    void* stream);
int rb_nvfp4_swiglu_backward_strided(const void* grad_h, int64_t ldgh, const void* gate, const void* up, int64_t ld,
                                     int64_t blk, int64_t rows, int64_t hidden, void* grad_gate, void* grad_up,
                                     int64_t ldo, int64_t blko, float* gs_out, void* workspace, void* stream);

/*
 * Test aid: the SwiGLU epilogue takes silu(g), rounded to bf16, from a table and three closed forms
 * instead of evaluating g / (1 + exp(-g)) per element; this checks that mapping on all 65536 bf16
 * bit patterns g against bf16 of the IEEE evaluation.  mismatches: 2 device uint32 (zeroed by the
 * caller); [0] counts the inputs whose bf16 results differ, [1] is the largest failing bit pattern
 * plus one (0 if none).
 */
int rb_nvfp4_selftest_silu(uint32_t* mismatches, void* stream);

/*
 * Global scale and column sums of x in one read: *gs_out as rb_nvfp4_global_scale computes it, and
 * colsum_out[c] = sum over rows of x[r, c] (fp32 accumulation in a fixed order, so repeated calls
 * agree bit for bit).  For the upstream gradient of a linear with a bias, whose quantization needs
 * gs and whose bias gradient is dY.sum(0) (linear.py:146-147 in jamespa16/radiance: a separate torch
 * reduction there, a second full read of dY).
 *   x          : rows x cols of `dtype`, row stride ld elements; 16-byte aligned base, cols*elemsize
 *                and ld*elemsize multiples of 16.
 *   colsum_out : device fp32[cols].
 *   workspace  : rb_nvfp4_global_scale_colsum_workspace(dtype, rows, cols) bytes, 16-byte aligned;
 *                its first 16 bytes zeroed before the first call (every call leaves them zeroed
 *                again, so calls ordered on one stream can share it).
 */
size_t rb_nvfp4_global_scale_colsum_workspace(int dtype, int64_t rows, int64_t cols);
int rb_nvfp4_global_scale_colsum(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* gs_out,
                                 float* colsum_out, void* workspace, void* stream);

/*
 * Grouped (mixture-of-experts) GEMMs, global scales and quantization.  radiance runs its experts
 * as stacked bf16 batched matmuls (BatchedExperts.forward, src/radiance/model/ffn.py:148-153:
 * torch.baddbmm over (experts, capacity, d)) and has no FP4 expert path (transformer.py:204-213
 * rejects FP4 + MoE); these entries give that path NVFP4 operands.  A group is a contiguous row
 * range of one stacked tensor: the tokens routed to one expert, or one expert's weight.
 *
 * Per-group global scales: gs_out[g] = max(amax(|x[offsets[g] : offsets[g+1]]|) / 2688, 1e-12)
 * (global_scale_of, quantize.py:205-213, per group; an empty group gets 1e-12).
 *   offsets   : device int64[num_groups + 1], non-decreasing, offsets[0] = 0, offsets[num_groups] <= rows.
 *   workspace : device uint32[num_groups + 1], zero before the first call; left zero again.
 *   cols * elemsize and ld * elemsize multiples of 16, x 16-byte aligned.
 */
int rb_nvfp4_global_scale_grouped(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                  const int64_t* offsets, int num_groups, float* gs_out, void* workspace,
                                  void* stream);

/*
 * rb_nvfp4_quantize with one global scale per group: every 128-row tile is quantized with
 * group_gs[g] for the group g that holds its first row.  With group offsets that are multiples of
 * 128 each group's rows of the outputs equal rb_nvfp4_quantize of that group alone (its packed
 * rows and scale tiles sit at the group's row offset of the rowblock outputs, at its column
 * offset of the colblock outputs).  Same shape contract and output sizes as rb_nvfp4_quantize.
 */
int rb_nvfp4_quantize_grouped(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                              const int64_t* offsets, int num_groups, const float* group_gs, const float* hadamard,
                              const int64_t* seed, void* row_packed, void* row_scale, void* col_packed,
                              void* col_scale, void* stream);

/*
 * Grouped block-scaled GEMM: for every group g with the device record
 *   groups[6g .. 6g+5] = {a_row0, b_row0, out_row0, m, k0, k}
 *   out[out_row0 + i, j] = alpha_a[g] * alpha_b[g] * sum_{k0 <= c < k0 + k} deq(a)[a_row0 + i, c] * deq(b)[b_row0 + j, c]
 * for i < m, j < n.  One launch covers all groups; the records stay on the device (no host sync
 * on routing counts).  a (a_rows rows) and b (b_rows rows) are rowblock-layout operands over one
 * contraction axis of k_total elements (their scale grids are k_total/64 blocks wide); out has
 * out_rows rows of n `out_dtype` elements, row stride ldo.  Forward and dgrad of an expert layer
 * are groups over token rows (k0 = 0, k = k_total); its wgrad is groups over contraction ranges
 * (the experts' token ranges of colblock-quantized operands).
 *   Device-side contract per record: a_row0, b_row0, m multiples of 128; k0, k multiples of 64;
 *   k0 + k <= k_total.  A record that breaks it is skipped and rb_nvfp4_device_status reports 5.
 *   A group with k == 0 writes zeros.  Rows past a group's m (up to the next multiple of 256) are
 *   computed but not stored.
 *   alpha_a, alpha_b : NULL or device fp32[num_groups].
 *   a_rows, b_rows, n multiples of 128; k_total multiple of 64; num_groups <= 256.
 */
int rb_nvfp4_gemm_grouped(const void* a_packed, const void* a_scale, int64_t a_rows, const void* b_packed,
                          const void* b_scale, int64_t b_rows, int64_t n, int64_t k_total, const int64_t* groups,
                          int num_groups, const float* alpha_a, const float* alpha_b, void* out, int out_dtype,
                          int64_t out_rows, int64_t ldo, void* stream);

/*
 * Self-test of the quantizer's division: for i < n, compares the library's correctly rounded
 * quotient x[i] / d[i] (reciprocal plus two residual corrections) with the IEEE quotient and
 * counts mismatching bit patterns into *mismatches (device uint32, accumulated).  Test aid; no
 * counterpart in the reference.
 */
int rb_nvfp4_selftest_division(const float* x, const float* d, int64_t n, uint32_t* mismatches, void* stream);

/*
 * Self-test of the quantizer's block-scale shortcut: for i < n, compares the scale byte the
 * quantizer derives for a block amax of amax[i] (a hardware e4m3 rounding of amax / (6 gs) and one
 * per-CTA threshold) with the exact evaluation (correctly rounded quotient, clamp, round up to
 * e4m3), under the device fp32 global scale *gs, and counts mismatches into *mismatches (device
 * uint32, accumulated).  Test aid; no counterpart in the reference.
 */
int rb_nvfp4_selftest_scale(const float* amax, int64_t n, const float* gs, uint32_t* mismatches, void* stream);

/*
 * Self-test of the failure path: launches one CTA that waits, with the library's bounded mbarrier
 * wait shortened to limit_cycles (0 < limit_cycles <= the ~1 s production limit), on a barrier that
 * nothing ever arrives on.  No TMA copy, MMA or TMEM allocation is issued, so nothing is in flight
 * when the wait gives up; the kernel then records the status a real timeout records and returns.
 *   which = 0 : the quantizer's wait (status 1, TMA data), recorded in the quantizer's status word;
 *   which = 1 : the GEMM epilogue's sleeping wait (status 2, MMA completion), in the GEMM's word.
 *   waited_cycles : device uint32, set to the cycles the wait took before giving up.
 * rb_nvfp4_device_status then reports the code, and later launches run normally.  Test aid; no
 * counterpart in the reference.
 */
int rb_nvfp4_selftest_wait_timeout(int which, long long limit_cycles, uint32_t* waited_cycles, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RADIANCE_NVFP4_H_ */
