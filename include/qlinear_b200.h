/*
 * qlinear_b200.h -- C ABI of the B200 (sm_100a) quantized-linear kernels.
 *
 * Drop-in boundary for the quantized-linear hot path of the ComfyUI
 * INT8-Fast node pack (reference v1.3.4).  The reference is pure Python: its
 * kernels are Triton functions called from PyTorch.  Each entry point below
 * replaces one of them (or one PyTorch expression on the hot path); the
 * comment on each cites the reference interface it replaces.  The Python
 * package binds these with ctypes (_native.py).
 *
 * Conventions
 *  - All pointers are device pointers unless stated otherwise; matrices are
 *    row-major with the given leading dimension (in elements).
 *  - `stream` is a cudaStream_t (NULL = legacy default stream); work is
 *    enqueued asynchronously on it, nothing synchronises the host.
 *  - The device is the calling thread's current CUDA device.
 *  - Every function returns QLIN_OK (0) or a QLIN_ERR_* code and never throws;
 *    qlin_last_error() returns a thread-local message for the last failure.
 *  - Numerics follow the reference's PyTorch CPU path bit for bit (codes,
 *    scales, int32 accumulators, and outputs of the reference's epilogues);
 *    each GEMM entry point below states its epilogue's rounding order.  The
 *    exceptions are stated where they occur: the ConvRot rotation sums in a
 *    fixed butterfly order (the reference's library matmul has its own), the
 *    GELU step of qlin_gemm_w8a8_fused is within one unit of out_dtype of the
 *    exact function, and the group-128 schemes have no reference at all.
 */
#ifndef QLINEAR_B200_H
#define QLINEAR_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define QLIN_API __attribute__((visibility("default")))
#else
#define QLIN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define QLIN_OK 0
#define QLIN_ERR_INVALID_ARG 1   /* bad shape / null pointer / enum value      */
#define QLIN_ERR_UNSUPPORTED 2   /* valid request this build does not handle   */
#define QLIN_ERR_ALIGNMENT 3     /* pointer or leading dimension misaligned    */
#define QLIN_ERR_CUDA 4          /* a CUDA runtime/driver call failed          */
#define QLIN_ERR_NO_DEVICE 5     /* current device is not an sm_100 GPU        */

/* element types */
#define QLIN_BF16 0
#define QLIN_F16 1
#define QLIN_F32 2
#define QLIN_I8 3
#define QLIN_I32 4

/* Hadamard families for ConvRot */
#define QLIN_ROT_NONE 0
#define QLIN_ROT_REGULAR 1   /* H4 (x) ... (x) H4, sizes 16, 64, 256 (convrot.py:18-55)        */
#define QLIN_ROT_SYLVESTER 2 /* Sylvester H2^(x)k, sizes 32 and 128 (scipy.linalg.hadamard)  */

/* weight-scale layouts for the W8A8 epilogue */
#define QLIN_WSCALE_TENSOR 0 /* one float: int8_quant.py:113-133 order (ws*xs) */
#define QLIN_WSCALE_ROW 1    /* float[N]:  int8_quant.py:137-164 order (xs then ws) */

/* row norms of the fused activation prologue */
#define QLIN_NORM_NONE 0
#define QLIN_NORM_LAYER 1  /* (x - mean) * rsqrt(var + eps), no affine: F.layer_norm(x, (K,), eps=eps) */
#define QLIN_NORM_RMS 2    /* dt((x * rsqrt(mean(x^2) + eps)) * weight): F.rms_norm(x, (K,), weight, eps) */

/* rounding modes for weight requantisation */
#define QLIN_ROUND_NEAREST 0    /* quantize_int8 (int8_quant.py:41-42)             */
#define QLIN_ROUND_STOCHASTIC 1 /* stochastic_round_int8_delta (int8_quant.py:80-106) */

/* Library identification and diagnostics. */
QLIN_API int qlin_version(void);
/* Makes `device` current for the calling thread (the entry points below run
 * on the current device; callers that switch devices call this first). */
QLIN_API int qlin_set_device(int device);
QLIN_API const char* qlin_last_error(void);
/* Reads and clears the device-side error words of the current device (bit 0:
 * a pipeline wait inside a GEMM kernel timed out; bit 1: a row kernel's
 * bulk-copy wait timed out; bit 2: after a GEMM timeout its in-flight work
 * did not drain within the limit; bit 3: a split-K GEMM found its scratch
 * counters non-zero on entry).  Synchronises `stream`. */
QLIN_API int qlin_device_error(void* stream, uint32_t* error_bits);

/* ---- failure detection ---------------------------------------------------
 * Every pipeline wait inside the kernels is bounded.  When a wait makes no
 * progress for the limit, the kernel sets a bit of the device error word,
 * every role of the CTA leaves its loop, the GEMM's in-flight TMA loads and
 * MMAs are drained (bit 2 if that drain also runs out), tensor memory is
 * released and the kernel returns; the context stays usable.  No
 * counterpart in the reference, which has no device-side error reporting
 * (its only error handling is host-side ValueErrors,
 * rocm_int8_kitchen_patch.py:138-150). */

/* Sets the wait limit of the current device's kernels, in nanoseconds
 * (1 us .. 60 s; 0 restores the default of 2 s).  Synchronous. */
QLIN_API int qlin_set_wait_limit(uint64_t limit_ns);

/* Self-test of the bounded wait: one thread waits on an mbarrier phase that
 * nothing completes, for the current limit, then returns.  which 0: the
 * GEMM pipeline wait (sets error bit 0); which 1: the row kernels' wait
 * (sets error bit 1). */
QLIN_API int qlin_selftest_wait_timeout(int which, void* stream);

/* Self-test of a whole GEMM's abort path: the W8A8 per-row GEMM with bf16
 * output and no bias (as qlin_gemm_w8a8) whose TMA producer leaves K-slab
 * `stall_kb` (128 int8 of K) of each CTA's first tile unfilled, so the MMA
 * issuer's wait for it runs out after the limit: error bit 0 is set and the
 * kernel returns with `out` partly written. */
QLIN_API int qlin_selftest_gemm_stall(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                      void* out, int64_t M, int64_t N, int64_t K, int64_t stall_kb, void* stream);

/* ---- (a) activation quantisation, fused with the ConvRot rotation -------- */

/* Per-token int8 quantisation of x[M,K] (dtype x_dtype in {BF16,F16,F32}),
 * optionally preceded by the block-diagonal Hadamard rotation of group
 * `rot_group` (rot_kind != QLIN_ROT_NONE), rounded to x_dtype before
 * quantising.  Writes q[M,K] int8 (row stride K) and scale[M] float.
 * rot_c is the +-entry of the normalised Hadamard in x_dtype.
 * Replaces: triton_quantize_rowwise (int8_fused_kernel.py:67-85) and the
 * PyTorch quantize_int8_axiswise(x, dim=-1) (int8_quant.py:49-52), fused
 * with rotate_activation (convrot.py:89-118, called at int8_quant.py:702-706). */
QLIN_API int qlin_quant_act_int8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                 int rot_kind, int rot_group, float rot_c,
                                 int8_t* q, float* scale, void* stream);

/* qlin_quant_act_int8 preceded by a DiT block's row norm and modulation,
 * each step rounded to x_dtype as the eager PyTorch sequence rounds it:
 *   y = dt(norm(x))                          norm_kind QLIN_NORM_* (float32 row statistics,
 *                                            rsqrt correctly rounded), norm_weight [K] or NULL
 *   y = dt(y * mod_mul[s, :])                if mod_mul (e.g. 1 + scale of a Flux modulation)
 *   y = dt(y + mod_add[s, :])                if mod_add (the shift)
 * with s = row / rows_per_sample (rows_per_sample <= 0: one sample),
 * mod_mul rows mul_ld and mod_add rows add_ld elements apart (rows
 * 0 .. (M-1)/rows_per_sample must exist); then the optional rotation and the
 * per-token int8 quantisation of qlin_quant_act_int8 on y.
 * x_dtype BF16 or F16; K % 16 == 0 (K <= 32768); x rows, q, norm_weight and
 * every mod_* row 16-byte aligned.
 * Replaces the eager prologue of the quantised linear: the kitchen
 * input_act RMS norm (rocm_int8_kitchen_patch.py:136) and a DiT block's
 * LayerNorm + (1 + scale) * x + shift in front of Int8TensorwiseOps.Linear
 * (int8_quant.py:633-716); the rows' statistics are summed in float32 in a
 * fixed order, which the eager kernels do in their own order. */
QLIN_API int qlin_quant_act_int8_norm(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                      int norm_kind, float eps, const void* norm_weight,
                                      const void* mod_mul, int64_t mul_ld, const void* mod_add,
                                      int64_t add_ld, int64_t rows_per_sample, int rot_kind, int rot_group, float rot_c,
                                      int8_t* q, float* scale, void* stream);

/* qlin_quant_act_int8 of concatenated rows: row r of the quantised input is
 * [x1[r, 0:K1] | x2[r, 0:K2]] (K = K1 + K2), x1 rows ld1 and x2 rows ld2
 * elements apart, so the concatenation is never written to memory.
 * x_dtype BF16, F16 or F32; K1 and K2 multiples of 16 (K <= 32768); both
 * sources and both row strides 16-byte aligned; q [M, K], scale [M].
 * Replaces the torch.cat that feeds a quantised linear, e.g. a Flux single
 * block's linear2(cat(attention, mlp_act(mlp))) in front of
 * Int8TensorwiseOps.Linear (int8_quant.py:633-716); no counterpart in the
 * reference's own files, which leave the model code to ComfyUI. */
QLIN_API int qlin_quant_act_int8_cat(const void* x1, int64_t ld1, int64_t K1, const void* x2, int64_t ld2,
                                     int64_t K2, int x_dtype, int64_t M, int rot_kind, int rot_group, float rot_c,
                                     int8_t* q, float* scale, void* stream);

/* Attention prologue of a Flux-style DiT block, in place on the fused qkv
 * projection: rows [rows, ld] in dtype (BF16 or F16), each row holding
 * `heads` q vectors, then `heads` k vectors, then the v vectors, head_dim
 * (64 or 128) elements each.  For every q and k vector x:
 *   n = dt((x * rsqrt(mean(x^2) + eps)) * w)     (F.rms_norm; w = q_weight or
 *                                                 k_weight [head_dim], NULL = none)
 * then, when cos_tab / sin_tab are given (float32 [positions, head_dim/2],
 * table row = row % positions), each pair (a, b) = (n[2i], n[2i+1]) becomes
 *   (dt(c*a - s*b), dt(s*a + c*b))               (each float32 product and sum rounded)
 * with c = cos_tab[pos, i], s = sin_tab[pos, i].  v is not touched.
 * qkv, ld * element size, the weights and the tables 16-byte aligned;
 * ld >= 2 * heads * head_dim.  No counterpart in the reference (the model
 * code around its quantised linears lives in ComfyUI); replaces the eager
 * q/k RMSNorm and rotary embedding between a DiT block's quantised qkv
 * linear and its attention. */
QLIN_API int qlin_qk_norm_rope(void* qkv, int dtype, int64_t rows, int64_t ld, int heads, int head_dim,
                               const void* q_weight, const void* k_weight, float eps, const float* cos_tab,
                               const float* sin_tab, int64_t positions, void* stream);

/* Signed int4-range quantisation (codes in [-7,7], one per int8 byte) with
 * the int4_quant.py conventions computed in x_dtype: absmax clamped at
 * clamp_min (1e-10 in x_dtype), scale = absmax/7, round(x/scale).
 * group == 0: per row, scale[M]   (quantize_signed_int4_rowwise, int4_quant.py:65-73)
 * group == 128: per row and K-group, scale[M, K/128] (group-128 scheme).
 * Optional fused rotation as above (prepare_rotated_activation, int4_quant.py:255-289). */
QLIN_API int qlin_quant_act_int4(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                                 int rot_kind, int rot_group, float rot_c, int group, float clamp_min,
                                 int8_t* q, float* scale, void* stream);

/* Rotation only: out[M,K] (x_dtype, row stride K) = rotate_activation(x)
 * (convrot.py:89-118); for float32 input this is rotate_weight (convrot.py:58-86). */
QLIN_API int qlin_rotate(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                         int rot_kind, int rot_group, float rot_c, void* out, void* stream);

/* SiTU gated input activation: x[M, 2K] = [hidden | gate] (row stride ldx)
 * -> out[M, K] = 4 tanh(gate/4) * sigmoid(gate) * 25 tanh(hidden/25),
 * float32 math, result in x_dtype.  Replaces triton_situ
 * (int8_fused_kernel.py:389-440), the input_act="situ" prologue of
 * rocm_int8_linear (rocm_int8_kitchen_patch.py:131-133). */
QLIN_API int qlin_situ(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, void* out, void* stream);

/* qlin_situ followed by qlin_quant_act_int8 in one kernel: row r of the
 * quantised input is dt(situ(hidden[r], gate[r])) for x[M, 2K] =
 * [hidden | gate] (row stride ldx >= 2K), optionally rotated; the [M, K]
 * activation is never written to memory.  Codes and scales are bit-equal
 * to the two-call sequence.  x_dtype BF16 or F16; K a multiple of 16
 * (K <= 32768); x and the row stride 16-byte aligned; q [M, K], scale [M].
 * Replaces the input_act="situ" prologue plus the activation quantisation
 * of rocm_int8_linear (rocm_int8_kitchen_patch.py:131-171;
 * int8_fused_kernel.py:389-440 then :23-85). */
QLIN_API int qlin_quant_act_int8_situ(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int rot_kind,
                                      int rot_group, float rot_c, int8_t* q, float* scale, void* stream);

/* ---- (b) W8A8 GEMM on tcgen05 kind::i8 ------------------------------------ */

/* out[M,N] = epilogue( a[M,K] int8 . w[N,K]^T int8 ) with int32 accumulation.
 * wscale_mode QLIN_WSCALE_ROW:    out = dt(dt(float(acc)*a_scale[m]*w_scale[n]) + bias[n])
 * wscale_mode QLIN_WSCALE_TENSOR: out = dt(dt(float(acc)*(w_scale[0]*a_scale[m])) + bias[n])
 * (dt = out_dtype rounding; bias has out_dtype, may be NULL.)
 * K % 16 == 0; a, w 16-byte aligned.
 * Replaces: triton_int8_linear_per_row / triton_int8_linear
 * (int8_fused_kernel.py:332-377, 184-244) with the epilogue order of the
 * PyTorch path int8_forward_dynamic_per_row / int8_forward_dynamic
 * (int8_quant.py:137-164, 113-133). */
QLIN_API int qlin_gemm_w8a8(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                            int wscale_mode, const void* bias, void* out, int out_dtype,
                            int64_t M, int64_t N, int64_t K, void* stream);

/* qlin_gemm_w8a8 with the K dimension split over CTA pairs, for problems
 * whose 256 x 256 output tiles leave most of the GPU idle (e.g. M = 1024,
 * N = 3072): each tile's K range is cut into up to 3 parts that run on
 * different CTA pairs; the parts meet through int32 partials in `scratch`
 * and the last one to finish adds them (exact integer sums) and runs the
 * qlin_gemm_w8a8 epilogue, so the output is bit-identical to qlin_gemm_w8a8.
 * qlin_gemm_w8a8_splitk_scratch gives the scratch size for a problem on the
 * current device (0: no split pays; qlin_gemm_w8a8_splitk then runs the
 * unsplit kernel and needs no scratch).  scratch: that many bytes of device
 * memory, 256-byte aligned, whose first 64 KB (counters and flags, at the
 * same place for every problem size) are zero before its first use; every
 * complete call leaves them zero again, so one scratch buffer serves calls
 * of any shape in turn.  Calls that share one scratch must not overlap on
 * the GPU.  Counters found non-zero on entry set bit 3 (value 8) of the
 * device error word (qlin_device_error) and the call writes no output.
 * Replaces: the reference's one-kernel triton_int8_linear(_per_row)
 * launch (int8_fused_kernel.py:332-377), whose grid is one program per
 * 128 x 256 output tile at any size. */
QLIN_API int qlin_gemm_w8a8_splitk_scratch(int64_t M, int64_t N, int64_t K, uint64_t* bytes);
QLIN_API int qlin_gemm_w8a8_splitk(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                   int wscale_mode, const void* bias, void* out, int out_dtype,
                                   int64_t M, int64_t N, int64_t K, void* scratch, uint64_t scratch_bytes,
                                   void* stream);

/* qlin_gemm_w8a8_splitk for callers that cannot allocate device memory when
 * they run the GEMM (an engine that reserves its GPU memory up front and
 * forbids later allocations, a plugin host that owns the allocator and
 * passes only input and output buffers): the split-K scratch is a fixed
 * 16 MiB array inside this library's device image instead of a
 * caller-provided buffer.  This call allocates nothing.  Every GPU that
 * loads the library holds that array until the process exits.  A problem
 * whose split needs more than the array holds is refused with
 * QLIN_ERR_UNSUPPORTED (on a 148-SM B200 every split plan fits: at most
 * 12.1 MiB).  The first call on each device looks the array's address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Each split call clears the array's counters first (cudaMemsetAsync on
 * `stream`).  All calls share the one array: calls that overlap on the GPU
 * (several streams or host threads) race on it and must be serialised by
 * the caller.  Same arguments and output bits as qlin_gemm_w8a8.  No
 * counterpart in the reference. */
QLIN_API int qlin_gemm_w8a8_splitk_noalloc(const int8_t* a, const float* a_scale, const int8_t* w,
                                           const float* w_scale, int wscale_mode, const void* bias, void* out,
                                           int out_dtype, int64_t M, int64_t N, int64_t K, void* stream);

/* qlin_gemm_w8a8 followed, inside the epilogue, by the element-wise steps
 * that follow a DiT block's linears (out_dtype BF16 or F16; y = the
 * qlin_gemm_w8a8 value, already rounded to out_dtype):
 *   y = dt(gelu_tanh(y))                       columns >= gelu_col0 (gelu_col0 >= N: none)
 *   y = dt(residual + dt(gate[g, n] * y))      if residual; without gate dt(residual + y)
 * with g = row / rows_per_gate (<= 0: one gate row; gate rows
 * 0 .. (M-1)/rows_per_gate must exist), residual [M, ld_res] and gate rows
 * gate_ld elements apart, both in out_dtype, 16-byte aligned rows.
 * gelu_tanh is F.gelu(approximate="tanh"), 0.5 y (1 + tanh(u)), evaluated
 * as the equal y * sigmoid(2u) in float32 with the special-function unit's
 * exp2 and reciprocal: within one unit of out_dtype of the exact function
 * (eager PyTorch's tanh form loses accuracy where 1 + tanh(u) cancels).
 * Replaces: the kitchen residual form residual + residual_scale * linear(x)
 * (rocm_int8_kitchen_patch.py:176) and a DiT block's gated residual
 * x + gate * linear(h) / GELU after Int8TensorwiseOps.Linear. */
QLIN_API int qlin_gemm_w8a8_fused(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                  int wscale_mode, const void* bias, void* out, int out_dtype,
                                  int64_t M, int64_t N, int64_t K, int64_t gelu_col0,
                                  const void* residual, int64_t ld_res, const void* gate, int64_t gate_ld,
                                  int64_t rows_per_gate, void* stream);

/* qlin_gemm_w8a8_fused (GELU / gated residual steps optional: gelu_col0 >= N
 * and residual == NULL give the plain epilogue) with segmented rows: logical
 * row r of a and a_scale is row (r / a_seg_rows) * a_seg_stride + a_seg_off
 * of those arrays, and logical output row r is row (r / out_seg_rows) *
 * out_seg_stride + out_seg_off of out ([.., N] row-major); a zero row count
 * leaves that side contiguous.  Residual and gate rows stay logical.
 * a_seg_rows a multiple of 128, out_seg_rows of 32, each dividing M; every
 * segment inside its stride (offset + rows <= stride); M and N >= 256
 * (CTA-pair kernel).  No counterpart in the reference, whose linears take
 * contiguous rows: this lets the two streams of a Flux-style double block
 * write their q/k/v rows straight into the joint [text | image] sequence of
 * each sample, and read their output projections' rows from the joint
 * attention output, where a model otherwise runs torch.cat and slice
 * copies. */
QLIN_API int qlin_gemm_w8a8_fused_segments(const int8_t* a, const float* a_scale, const int8_t* w,
                                           const float* w_scale, int wscale_mode, const void* bias, void* out,
                                           int out_dtype, int64_t M, int64_t N, int64_t K, int64_t gelu_col0,
                                           const void* residual, int64_t ld_res, const void* gate, int64_t gate_ld,
                                           int64_t rows_per_gate, int64_t a_seg_rows, int64_t a_seg_stride,
                                           int64_t a_seg_off, int64_t out_seg_rows, int64_t out_seg_stride,
                                           int64_t out_seg_off, void* stream);

/* Tensor-parallel W8A8 linear fused with its all-gather: this rank's column
 * shard, out[:, col_off : col_off + N_shard] = the qlin_gemm_w8a8 result for
 * (a, a_scale, w_shard, w_scale_shard, bias_shard), is stored into each of
 * the n_out buffers out_bufs[0..n_out) -- [M, ldo] row-major in out_dtype,
 * typically the peer mappings of one symmetric allocation, so every rank
 * ends up with the whole [M, ldo] output without a separate collective.
 * out_bufs is a host array; 1 <= n_out <= 8; col_off + N_shard <= ldo;
 * every buffer, col_off and ldo 16-byte aligned in bytes.  The kernel ends
 * with a system-scope fence; the caller orders the peers' reads after the
 * stores with a cross-GPU barrier, and their previous reads of the buffers
 * before the call.  No counterpart in the reference, which runs on one
 * device: this is the column-split latency mode of a multi-GPU linear. */
QLIN_API int qlin_gemm_w8a8_allgather(const int8_t* a, const float* a_scale, const int8_t* w_shard,
                                      const float* w_scale_shard, int wscale_mode, const void* bias_shard,
                                      void* const* out_bufs, int n_out, int64_t col_off, int64_t ldo, int out_dtype,
                                      int64_t M, int64_t N_shard, int64_t K, void* stream);

/* c[M,N] int32 = a[M,K] . w[N,K]^T (torch._int_mm(a, w.T), int8_quant.py:124,152). */
QLIN_API int qlin_int_mm(const int8_t* a, const int8_t* w, int32_t* c,
                         int64_t M, int64_t N, int64_t K, void* stream);

/* ---- (c) packed-INT4 GEMMs (nibbles unpacked in shared memory) ------------ */

/* c[M,N] int32 = a[M,K] . unpack(w_packed[N,K/2])^T, signed nibbles, low
 * nibble = even k.  Replaces triton_int4_mm (triton_int4_mm.py:123-170). */
QLIN_API int qlin_int4_mm(const int8_t* a, const int8_t* w_packed, int32_t* c,
                          int64_t M, int64_t N, int64_t K, void* stream);

/* W4A4 per-row linear: out = dt(float(acc)*a_scale[m]*w_scale[n] + bias[n])
 * in float32 with one rounding (convrot_w4a4_forward, int4_quant.py:325-353);
 * bias has out_dtype (converted to float32), may be NULL. */
QLIN_API int qlin_gemm_w4a4(const int8_t* a, const float* a_scale, const int8_t* w_packed,
                            const float* w_scale, const void* bias, void* out, int out_dtype,
                            int64_t M, int64_t N, int64_t K, void* stream);

/* Group-128 W4A8 (int8 activations, per-token scale a_scale[M]; weights
 * packed int4 with bf16 scales w_gscale[N, K/128]):
 *   acc = 0; for g: acc = fmaf(float(P_g[m,n]), w_gscale[n,g], acc)
 *   out = dt(acc * a_scale[m] + bias[n])
 * Group-128 W4A4 (int4 activations with float scales a_gscale[M, K/128]):
 *   acc = fmaf(float(P_g), a_gscale[m,g]*w_gscale[n,g], acc); out = dt(acc + bias[n]).
 * No counterpart in the reference (it has per-row int4 only); these follow
 * the int4_quant.py conventions. */
QLIN_API int qlin_gemm_w4a8_g128(const int8_t* a, const float* a_scale, const int8_t* w_packed,
                                 const uint16_t* w_gscale_bf16, const void* bias, void* out, int out_dtype,
                                 int64_t M, int64_t N, int64_t K, void* stream);
QLIN_API int qlin_gemm_w4a4_g128(const int8_t* a, const float* a_gscale, const int8_t* w_packed,
                                 const uint16_t* w_gscale_bf16, const void* bias, void* out, int out_dtype,
                                 int64_t M, int64_t N, int64_t K, void* stream);

/* ---- (d) weight-side kernels for loaders and LoRA ------------------------- */

/* On-the-fly weight quantisation: w[N,K] (BF16/F16/F32) -> float32 ->
 * optional rotate_weight -> quantize_int8_axiswise(dim=1): q[N,K], scale[N].
 * Replaces int8_quant.py:527-554 (and 276-326). */
QLIN_API int qlin_quant_weight_int8(const void* w, int w_dtype, int64_t N, int64_t K,
                                    int rot_kind, int rot_group, float rot_c,
                                    int8_t* q, float* scale, void* stream);

/* ConvRot W4A4 weight quantisation, packed[N,K/2] (low nibble = even k):
 * group == 0: float32 -> rotate_weight -> quantize_signed_int4_rowwise_packed,
 *             scale[N] (quantize_convrot_w4a4_weight, int4_quant.py:121-134);
 * group == 128: the same conventions per 128-wide K group, computed in the
 *             weight's dtype, scale[N, K/128] (group-128 scheme). */
QLIN_API int qlin_quant_weight_int4(const void* w, int w_dtype, int64_t N, int64_t K,
                                    int rot_kind, int rot_group, float rot_c, int group,
                                    int8_t* packed, float* scale, void* stream);

/* Asymmetric W4A8 -> int8 per-channel: codebook[code]*s_channel[n]*s_rel[n,k/gs]
 * (w4a8_int8.py:46-75) followed by quantize_int8_axiswise(dim=1)
 * (int8_quant.py:679-687), in one pass.  s_rel is float8_e4m3fn bytes. */
QLIN_API int qlin_requant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                                    const uint8_t* s_rel_fp8, int group_size, int64_t N, int64_t K,
                                    int8_t* q, float* scale, void* stream);

/* Asymmetric W4A8 -> float32: out[N,K] = codebook[code]*s_channel[n]*s_rel[n,k/gs],
 * multiplied in that order, the same expression as qlin_requant_asym_w4a8
 * before its requantisation.  Replaces dequant_asym_w4a8_to_float
 * (w4a8_int8.py:46-75). */
QLIN_API int qlin_dequant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                                    const uint8_t* s_rel_fp8, int group_size, int64_t N, int64_t K, float* out,
                                    void* stream);

/* LoRA bake helpers (int8_quant.py:809-843, 881-941).
 * dequant: out[N,K] float32 = rotate_weight(q * scale)   (rotation optional)
 * requant: q[N,K] = round(rotate_weight(w) * (1/scale)) with the ORIGINAL
 *          scale; QLIN_ROUND_STOCHASTIC uses a counter-based RNG seeded by
 *          `seed` (same distribution as the reference, not the same stream).
 * scale_mode: QLIN_WSCALE_TENSOR (one float) or QLIN_WSCALE_ROW (float[N]). */
QLIN_API int qlin_dequant_int8(const int8_t* q, const float* scale, int scale_mode, int64_t N, int64_t K,
                               int rot_kind, int rot_group, float rot_c, float* out, void* stream);
QLIN_API int qlin_requant_int8(const float* w, const float* scale, int scale_mode, int64_t N, int64_t K,
                               int rot_kind, int rot_group, float rot_c, int round_mode, uint64_t seed,
                               int8_t* q, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QLINEAR_B200_H */
