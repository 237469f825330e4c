// Host-side declarations shared by the translation units of libqlinear_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace qlin {

// thread-local last-error message behind qlin_last_error()
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Number of SMs of the current device (cached per device); 0 on failure.
int device_sm_count();

// Programmatic dependent launch: a kernel launched by launch_pdl may be
// scheduled while the previous kernel of the stream is still running and
// does its set-up (barriers, TMEM, descriptor prefetch) meanwhile; every such
// kernel executes griddepcontrol.wait (pdl_wait) in all threads before its
// first global-memory access, which returns once the previous kernel has
// completed and its writes are visible.  QLIN_NO_PDL=1 launches in plain
// stream order.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// Major*10+minor of the current device (cached); 0 on failure.
int device_cc();

struct RowQuantLaunch {
  int dt_in;       // DT_BF16/F16/F32/I8
  int dt_q;        // compute dtype of rotation + quantisation
  int rot_kind;    // ROT_*
  int rot_group;   // 0 when rot_kind == ROT_NONE
  int mode;        // MODE_*
};

// Launch the row kernel family; returns a QLIN_* status.
int launch_rowquant(const RowQuantLaunch& L, const void* x, int64_t ldx, int64_t M, int64_t K, float rot_c,
                    float clamp_min, const float* in_scale, int in_scale_per_row, int8_t* q, float* scale,
                    void* out, uint64_t seed, cudaStream_t stream);

// Row norm + modulation prologue of the int8 activation quantiser (see
// RowQuantParams): norm_kind NORM_*, vectors in the input dtype.
struct FusedPrologue {
  int norm_kind;
  float eps;
  const void* norm_w;
  const void* mod_mul;
  int64_t mul_ld;
  const void* mod_add;
  int64_t add_ld;
  int64_t rows_per_sample;  // <= 0: one sample
};
int launch_rowquant_fused(int dt, int rot_kind, int rot_group, float rot_c, const void* x, int64_t ldx, int64_t M,
                          int64_t K, const FusedPrologue& f, int8_t* q, float* scale, cudaStream_t stream);

int launch_rowquant_situ(int dt, int rot_kind, int rot_group, float rot_c, const void* x, int64_t ldx, int64_t M,
                         int64_t K, int8_t* q, float* scale, cudaStream_t stream);

int launch_rowquant_cat(int dt, int rot_kind, int rot_group, float rot_c, const void* x1, int64_t ld1, int64_t K1,
                        const void* x2, int64_t ld2, int64_t K2, int64_t M, int8_t* q, float* scale,
                        cudaStream_t stream);

// In-place q/k RMSNorm + rotary embedding of fused qkv rows (dit.cu).
int launch_qk_norm_rope(int dt, void* qkv, int64_t rows, int64_t ld, int heads, int head_dim, const void* q_w,
                        const void* k_w, float eps, const float* cos_t, const float* sin_t, int64_t positions,
                        cudaStream_t stream);

int launch_rowquant_generic(int dt, int mode, const void* x, int64_t ldx, int64_t M, int64_t K, float clamp_min,
                            int8_t* q, float* scale, cudaStream_t stream);

enum GemmKind { GEMM_W8A8_ROW = 0, GEMM_W8A8_TENSOR = 1, GEMM_W4A4_ROW = 2, GEMM_I32 = 3 };

// Launch the tcgen05 GEMM; b_int4 selects packed-int4 B.
int launch_gemm(int kind, bool b_int4, const int8_t* a, const int8_t* b, const float* a_scale,
                const float* w_scale, const void* bias, void* out, int out_dt, int64_t M, int64_t N, int64_t K,
                cudaStream_t stream);

// Output destinations of a GEMM: one buffer, or the same [M, ldo] buffer on
// every rank of a tensor-parallel group (peer pointers), written at column
// col_off.
struct OutSpec {
  void* outs[8];
  int nout;
  int64_t col_off;
  int64_t ldo;
};
// Element-wise steps after the W8A8 epilogue (16-bit outputs, one
// destination): y = dt(gelu_tanh(y)) for columns >= gelu_col0, then
// y = dt(residual + dt(gate * y)) (or dt(residual + y) without a gate), gate
// row = output row / rows_per_gate.
struct EpiPost {
  int64_t gelu_col0;        // >= N: no GELU
  const void* residual;     // [M, ld_res] or null
  int64_t ld_res;
  const void* gate;         // [M / rows_per_gate, gate_ld] or null
  int64_t gate_ld;
  int64_t rows_per_gate;
};
// Segmented rows of a W8A8 GEMM (CTA-pair kernel, 16-bit output through
// TMA stores, one destination): logical row r of A and a_scale is row
// (r / a_rows) * a_stride + a_off of those arrays, logical output row r is
// row (r / o_rows) * o_stride + o_off of the output ([.., ldo]); a_rows /
// o_rows 0: contiguous.  a_rows a multiple of 128, o_rows of 32, M a
// multiple of each.  Lets the two streams of a DiT double block write their
// qkv rows straight into the joint sequence, and read their projections'
// rows from the joint attention output, instead of copying.
struct GemmSegments {
  int64_t a_rows, a_stride, a_off;
  int64_t o_rows, o_stride, o_off;
};
int launch_gemm_to(int kind, bool b_int4, const int8_t* a, const int8_t* b, const float* a_scale,
                   const float* w_scale, const void* bias, const OutSpec& o, int out_dt, int64_t M, int64_t N,
                   int64_t K, cudaStream_t stream, const EpiPost* post = nullptr, const GemmSegments* seg = nullptr);

// Split-K W8A8 GEMM on CTA pairs (GemmParams::splits): the scratch size a
// problem needs (0: it runs unsplit), and the launch, which falls back to
// launch_gemm when no split pays.  The scratch's counters are zero on entry
// and left zero by every complete launch.
size_t splitk_scratch_bytes(int64_t M, int64_t N, int64_t K);
int launch_gemm_splitk(int kind, const int8_t* a, const int8_t* b, const float* a_scale, const float* w_scale,
                       const void* bias, void* out, int out_dt, int64_t M, int64_t N, int64_t K, void* scratch,
                       size_t scratch_bytes, cudaStream_t stream);
// Bytes at the start of a split-K scratch holding its counters and flags.
size_t splitk_header_bytes();
// launch_gemm_splitk on the library's fixed device array instead of caller
// scratch (noalloc.cu); allocates nothing.
int launch_gemm_splitk_noalloc(int kind, const int8_t* a, const int8_t* b, const float* a_scale,
                               const float* w_scale, const void* bias, void* out, int out_dt, int64_t M, int64_t N,
                               int64_t K, cudaStream_t stream);

int launch_gemm_g128(bool a_int4_groups, const int8_t* a, const float* a_scale, const int8_t* w_packed,
                     const uint16_t* w_gscale, const void* bias, void* out, int out_dt, int64_t M, int64_t N,
                     int64_t K, cudaStream_t stream);

// Asymmetric W4A8 rows: int8 requantisation (q, scale), or with wout set the
// float32 dequantised rows only.
int launch_requant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                             const uint8_t* s_rel, int group_size, int64_t N, int64_t K, int8_t* q, float* scale,
                             float* wout, cudaStream_t stream);

int launch_situ(int dt, const void* x, int64_t ldx, int64_t M, int64_t K, void* y, cudaStream_t stream);

int read_device_error(cudaStream_t stream, uint32_t* bits);
// Failure detection: wait limits of the GEMM and row-kernel pipelines, the
// one-thread wait self-tests, and a W8A8 GEMM whose producer leaves K-slab
// stall_kb of each CTA's first tile unfilled.
int set_gemm_wait_limit(uint64_t ns);
int set_rowquant_wait_limit(uint64_t ns);
int launch_wait_selftest(cudaStream_t stream);
int launch_rowquant_wait_selftest(cudaStream_t stream);
int launch_gemm_stall(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, void* out,
                      int64_t M, int64_t N, int64_t K, int64_t stall_kb, cudaStream_t stream);
int read_rowquant_error(cudaStream_t stream, uint32_t* bits);

}  // namespace qlin
