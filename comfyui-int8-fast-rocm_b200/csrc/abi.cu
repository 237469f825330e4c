// extern "C" entry points of libqlinear_b200.so: argument validation, error
// reporting and dispatch to the kernel launchers.  Nothing here throws.
#include <cstdint>
#include <cstdlib>
#include <string>

#include "../../include/qlinear_b200.h"
#include "common.cuh"
#include "internal.h"
#include "rowquant.cuh"

#include <nvtx3/nvToolsExt.h>

namespace {
// One NVTX range per C-ABI call, named after the entry point (visible in
// Nsight Systems / Nsight Compute timelines; a few nanoseconds when no tool
// is attached).
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
}  // namespace
#define QLIN_RANGE() NvtxRange qlin_nvtx_range_(__func__)

namespace qlin {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }
int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}
int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return QLIN_ERR_CUDA;
}

namespace {
constexpr int kMaxDevices = 64;
int g_sms[kMaxDevices] = {0};
int g_cc[kMaxDevices] = {0};

int current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return (d >= 0 && d < kMaxDevices) ? d : -1;
}
}  // namespace

int device_sm_count() {
  const int d = current_device();
  if (d < 0) return 0;
  if (!g_sms[d]) cudaDeviceGetAttribute(&g_sms[d], cudaDevAttrMultiProcessorCount, d);
  return g_sms[d];
}
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("QLIN_NO_PDL");
    return !(v != nullptr && v[0] == '1');
  }();
  return on;
}
int device_cc() {
  const int d = current_device();
  if (d < 0) return 0;
  if (!g_cc[d]) {
    int ma = 0, mi = 0;
    cudaDeviceGetAttribute(&ma, cudaDevAttrComputeCapabilityMajor, d);
    cudaDeviceGetAttribute(&mi, cudaDevAttrComputeCapabilityMinor, d);
    g_cc[d] = ma * 10 + mi;
  }
  return g_cc[d];
}

}  // namespace qlin

using namespace qlin;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int esize(int dt) { return dt == QLIN_F32 ? 4 : (dt == QLIN_I8 ? 1 : 2); }
bool float_dt(int dt) { return dt == QLIN_BF16 || dt == QLIN_F16 || dt == QLIN_F32; }

// ``clamp(min=1e-10)`` on a tensor of dtype dt compares with 1e-10 in dt.
float clamp_min_for(int dt) {
  if (dt == QLIN_BF16) return __bfloat162float(__float2bfloat16_rn(1e-10f));
  if (dt == QLIN_F16) return __half2float(__float2half_rn(1e-10f));
  return 1e-10f;
}

int check_device() {
  const int cc = device_cc();
  if (cc == 0) return fail(QLIN_ERR_NO_DEVICE, "no current CUDA device");
  if (cc != 100)
    return fail(QLIN_ERR_NO_DEVICE,
                "kernels are built for sm_100a (B200); device has compute capability " + std::to_string(cc));
  return QLIN_OK;
}

int check_rot(int kind, int group, int64_t K) {
  if (kind == QLIN_ROT_NONE) return QLIN_OK;
  if (kind != QLIN_ROT_REGULAR && kind != QLIN_ROT_SYLVESTER) return fail(QLIN_ERR_INVALID_ARG, "bad rot_kind");
  if (group <= 0 || K % group != 0)
    return fail(QLIN_ERR_INVALID_ARG,
                "features " + std::to_string(K) + " not divisible by group_size " + std::to_string(group));
  return QLIN_OK;
}

// Rows usable by the vectorised kernels: 16-element multiples, 16-byte aligned.
bool rows_vec_ok(const void* x, int64_t K, int64_t ldx, int dt) {
  return (K % 16 == 0) && aligned16(x) && ((ldx * esize(dt)) % 16 == 0);
}

int gemm_common_checks(const int8_t* a, const void* w, int64_t M, int64_t N, int64_t K, int kmul) {
  if (M < 0 || N < 0 || K <= 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) return fail(QLIN_ERR_UNSUPPORTED, "dimension too large");
  if (K % kmul) return fail(QLIN_ERR_ALIGNMENT, "K must be a multiple of " + std::to_string(kmul));
  if (M == 0 || N == 0) return QLIN_OK;
  if (!a || !w) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(a) || !aligned16(w)) return fail(QLIN_ERR_ALIGNMENT, "operands must be 16-byte aligned");
  return check_device();
}

}  // namespace

extern "C" {

QLIN_API int qlin_version(void) { return 10000; }

QLIN_API int qlin_set_device(int device) {
  QLIN_RANGE();
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return QLIN_OK;
}

QLIN_API const char* qlin_last_error(void) { return t_last_error.c_str(); }

QLIN_API int qlin_device_error(void* stream, uint32_t* error_bits) {
  QLIN_RANGE();
  if (!error_bits) return fail(QLIN_ERR_INVALID_ARG, "error_bits is null");
  int rc = check_device();
  if (rc) return rc;
  uint32_t gemm_bits = 0, row_bits = 0;
  if ((rc = read_device_error(static_cast<cudaStream_t>(stream), &gemm_bits))) return rc;
  if ((rc = read_rowquant_error(static_cast<cudaStream_t>(stream), &row_bits))) return rc;
  *error_bits = gemm_bits | row_bits;
  return QLIN_OK;
}

QLIN_API int qlin_set_wait_limit(uint64_t limit_ns) {
  QLIN_RANGE();
  int rc = check_device();
  if (rc) return rc;
  if (limit_ns == 0) limit_ns = 2000000000ull;
  if (limit_ns < 1000ull || limit_ns > 60000000000ull)
    return fail(QLIN_ERR_INVALID_ARG, "wait limit must lie between 1 us and 60 s");
  if ((rc = set_gemm_wait_limit(limit_ns))) return rc;
  return set_rowquant_wait_limit(limit_ns);
}

QLIN_API int qlin_selftest_wait_timeout(int which, void* stream) {
  QLIN_RANGE();
  int rc = check_device();
  if (rc) return rc;
  if (which == 0) return launch_wait_selftest(static_cast<cudaStream_t>(stream));
  if (which == 1) return launch_rowquant_wait_selftest(static_cast<cudaStream_t>(stream));
  return fail(QLIN_ERR_INVALID_ARG, "which must be 0 (GEMM pipeline wait) or 1 (row-kernel wait)");
}

QLIN_API int qlin_selftest_gemm_stall(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                      void* out, int64_t M, int64_t N, int64_t K, int64_t stall_kb, void* stream) {
  QLIN_RANGE();
  if (!a || !a_scale || !w || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (K % 16) return fail(QLIN_ERR_ALIGNMENT, "K must be a multiple of 16");
  if (!aligned16(a) || !aligned16(w) || !aligned16(out)) return fail(QLIN_ERR_ALIGNMENT, "operands must be 16-byte aligned");
  int rc = check_device();
  if (rc) return rc;
  return launch_gemm_stall(a, a_scale, w, w_scale, out, M, N, K, stall_kb, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_act_int8(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int rot_kind,
                                 int rot_group, float rot_c, int8_t* q, float* scale, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < K) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(x_dtype)) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16, F16 or F32");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = rows_vec_ok(x, K, ldx, x_dtype) && aligned16(q);
  if (!vec) {
    if (rot_kind != QLIN_ROT_NONE)
      return fail(QLIN_ERR_ALIGNMENT, "rotation needs K % 16 == 0 and 16-byte aligned rows");
    return launch_rowquant_generic(x_dtype, MODE_INT8, x, ldx, M, K, 0.0f, q, scale, s);
  }
  RowQuantLaunch L{x_dtype, x_dtype, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, MODE_INT8};
  return launch_rowquant(L, x, ldx, M, K, rot_c, 0.0f, nullptr, 0, q, scale, nullptr, 0, s);
}

QLIN_API int qlin_quant_act_int8_norm(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int norm_kind,
                                      float eps, const void* norm_weight, const void* mod_mul, int64_t mul_ld,
                                      const void* mod_add, int64_t add_ld, int64_t rows_per_sample, int rot_kind, int rot_group,
                                      float rot_c, int8_t* q, float* scale, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < K) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (x_dtype != QLIN_BF16 && x_dtype != QLIN_F16) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16 or F16");
  if (norm_kind != QLIN_NORM_NONE && norm_kind != QLIN_NORM_LAYER && norm_kind != QLIN_NORM_RMS)
    return fail(QLIN_ERR_INVALID_ARG, "bad norm_kind");
  if (norm_weight != nullptr && norm_kind != QLIN_NORM_RMS)
    return fail(QLIN_ERR_INVALID_ARG, "norm_weight is taken by QLIN_NORM_RMS only");
  if (!(eps >= 0.0f)) return fail(QLIN_ERR_INVALID_ARG, "eps must be >= 0");
  if ((mod_mul && mul_ld < K) || (mod_add && add_ld < K)) return fail(QLIN_ERR_INVALID_ARG, "modulation row stride < K");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (!rows_vec_ok(x, K, ldx, x_dtype) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "the fused prologue needs K % 16 == 0 and 16-byte aligned rows");
  if ((norm_weight && !aligned16(norm_weight)) || (mod_mul && (!aligned16(mod_mul) || (mul_ld * 2) % 16)) ||
      (mod_add && (!aligned16(mod_add) || (add_ld * 2) % 16)))
    return fail(QLIN_ERR_ALIGNMENT, "norm weight and modulation rows must be 16-byte aligned");
  FusedPrologue f{norm_kind, eps, norm_weight, mod_mul, mul_ld, mod_add, add_ld, rows_per_sample};
  return launch_rowquant_fused(x_dtype, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, rot_c, x, ldx, M, K, f,
                               q, scale, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_act_int8_situ(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int rot_kind,
                                      int rot_group, float rot_c, int8_t* q, float* scale, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < 2 * K) return fail(QLIN_ERR_INVALID_ARG, "bad shape (rows are [hidden | gate], ldx >= 2K)");
  if (x_dtype != QLIN_BF16 && x_dtype != QLIN_F16) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16 or F16");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (K % 16 != 0 || !rows_vec_ok(x, 2 * K, ldx, x_dtype) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "the SiTU prologue needs K % 16 == 0 and 16-byte aligned rows");
  return launch_rowquant_situ(x_dtype, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, rot_c, x, ldx, M, K, q,
                              scale, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_act_int8_cat(const void* x1, int64_t ld1, int64_t K1, const void* x2, int64_t ld2,
                                     int64_t K2, int x_dtype, int64_t M, int rot_kind, int rot_group, float rot_c,
                                     int8_t* q, float* scale, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K1 <= 0 || K2 <= 0 || ld1 < K1 || ld2 < K2) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(x_dtype)) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16, F16 or F32");
  if (M == 0) return QLIN_OK;
  if (!x1 || !x2 || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K1 + K2))) return rc;
  if (!rows_vec_ok(x1, K1, ld1, x_dtype) || !rows_vec_ok(x2, K2, ld2, x_dtype) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "concatenated rows need K1, K2 % 16 == 0 and 16-byte aligned rows");
  return launch_rowquant_cat(x_dtype, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, rot_c, x1, ld1, K1, x2,
                             ld2, K2, M, q, scale, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_qk_norm_rope(void* qkv, int dtype, int64_t rows, int64_t ld, int heads, int head_dim,
                               const void* q_weight, const void* k_weight, float eps, const float* cos_tab,
                               const float* sin_tab, int64_t positions, void* stream) {
  QLIN_RANGE();
  if (rows < 0 || heads < 0 || positions < 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (dtype != QLIN_BF16 && dtype != QLIN_F16) return fail(QLIN_ERR_INVALID_ARG, "dtype must be BF16 or F16");
  if (head_dim != 64 && head_dim != 128) return fail(QLIN_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (ld < 2 * (int64_t)heads * head_dim) return fail(QLIN_ERR_INVALID_ARG, "row stride shorter than the q and k heads");
  if (!(eps >= 0.0f)) return fail(QLIN_ERR_INVALID_ARG, "eps must be >= 0");
  if ((cos_tab == nullptr) != (sin_tab == nullptr)) return fail(QLIN_ERR_INVALID_ARG, "give both cos and sin tables");
  if (cos_tab && positions == 0) return fail(QLIN_ERR_INVALID_ARG, "the rotary tables need positions > 0");
  if (rows == 0 || heads == 0) return QLIN_OK;
  if (!qkv) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if (!aligned16(qkv) || (ld * 2) % 16 || (q_weight && !aligned16(q_weight)) || (k_weight && !aligned16(k_weight)) ||
      (cos_tab && (!aligned16(cos_tab) || !aligned16(sin_tab))))
    return fail(QLIN_ERR_ALIGNMENT, "qkv rows, norm weights and rotary tables must be 16-byte aligned");
  return launch_qk_norm_rope(dtype, qkv, rows, ld, heads, head_dim, q_weight, k_weight, eps, cos_tab, sin_tab,
                             positions, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_act_int4(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int rot_kind,
                                 int rot_group, float rot_c, int group, float clamp_min, int8_t* q, float* scale,
                                 void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < K) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(x_dtype)) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16, F16 or F32");
  if (group != 0 && group != 128) return fail(QLIN_ERR_UNSUPPORTED, "int4 group must be 0 (per row) or 128");
  if (group == 128 && K % 128) return fail(QLIN_ERR_INVALID_ARG, "K must be a multiple of 128 for group-128 int4");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = rows_vec_ok(x, K, ldx, x_dtype) && aligned16(q);
  if (!vec) {
    if (rot_kind != QLIN_ROT_NONE || group)
      return fail(QLIN_ERR_ALIGNMENT, "rotation / grouping needs K % 16 == 0 and 16-byte aligned rows");
    return launch_rowquant_generic(x_dtype, MODE_INT4_ROW, x, ldx, M, K, clamp_min, q, scale, s);
  }
  RowQuantLaunch L{x_dtype, x_dtype, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group,
                   group ? MODE_INT4_G128 : MODE_INT4_ROW};
  return launch_rowquant(L, x, ldx, M, K, rot_c, clamp_min, nullptr, 0, q, scale, nullptr, 0, s);
}

QLIN_API int qlin_rotate(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int rot_kind,
                         int rot_group, float rot_c, void* out, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < K) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(x_dtype)) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16, F16 or F32");
  if (rot_kind == QLIN_ROT_NONE) return fail(QLIN_ERR_INVALID_ARG, "qlin_rotate needs a rotation");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (!rows_vec_ok(x, K, ldx, x_dtype) || !aligned16(out))
    return fail(QLIN_ERR_ALIGNMENT, "rotation needs K % 16 == 0 and 16-byte aligned rows");
  RowQuantLaunch L{x_dtype, x_dtype, rot_kind, rot_group, MODE_ROTATE};
  return launch_rowquant(L, x, ldx, M, K, rot_c, 0.0f, nullptr, 0, nullptr, nullptr, out, 0,
                         static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w8a8(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                            int wscale_mode, const void* bias, void* out, int out_dtype, int64_t M, int64_t N,
                            int64_t K, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  return launch_gemm(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, false, a, w, a_scale,
                     w_scale, bias, out, out_dtype, M, N, K, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w8a8_splitk_scratch(int64_t M, int64_t N, int64_t K, uint64_t* bytes) {
  QLIN_RANGE();
  if (!bytes) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (M < 0 || N < 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(QLIN_ERR_INVALID_ARG, "bad GEMM shape");
  *bytes = (uint64_t)splitk_scratch_bytes(M, N, K);
  return QLIN_OK;
}

QLIN_API int qlin_gemm_w8a8_splitk(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                   int wscale_mode, const void* bias, void* out, int out_dtype, int64_t M, int64_t N,
                                   int64_t K, void* scratch, uint64_t scratch_bytes, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  return launch_gemm_splitk(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, a, w, a_scale, w_scale,
                            bias, out, out_dtype, M, N, K, scratch, (size_t)scratch_bytes,
                            static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w8a8_splitk_noalloc(const int8_t* a, const float* a_scale, const int8_t* w,
                                           const float* w_scale, int wscale_mode, const void* bias, void* out,
                                           int out_dtype, int64_t M, int64_t N, int64_t K, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  return launch_gemm_splitk_noalloc(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, a, w, a_scale,
                                    w_scale, bias, out, out_dtype, M, N, K, static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w8a8_fused(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                  int wscale_mode, const void* bias, void* out, int out_dtype, int64_t M, int64_t N,
                                  int64_t K, int64_t gelu_col0, const void* residual, int64_t ld_res,
                                  const void* gate, int64_t gate_ld, int64_t rows_per_gate, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (out_dtype != QLIN_BF16 && out_dtype != QLIN_F16)
    return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16 or F16 for the fused epilogue");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  if (gelu_col0 < 0) return fail(QLIN_ERR_INVALID_ARG, "gelu_col0 < 0");
  if (gate && !residual) return fail(QLIN_ERR_INVALID_ARG, "a gate needs a residual");
  if (residual && ld_res < N) return fail(QLIN_ERR_INVALID_ARG, "ld_res < N");
  if (gate && gate_ld < N) return fail(QLIN_ERR_INVALID_ARG, "gate_ld < N");
  if ((residual && (!aligned16(residual) || (ld_res * 2) % 16)) || (gate && (!aligned16(gate) || (gate_ld * 2) % 16)))
    return fail(QLIN_ERR_ALIGNMENT, "residual and gate rows must be 16-byte aligned");
  if (N % 8) return fail(QLIN_ERR_ALIGNMENT, "the fused epilogue needs N % 8 == 0");
  OutSpec o;
  for (int i = 0; i < 8; ++i) o.outs[i] = nullptr;
  o.outs[0] = out;
  o.nout = 1;
  o.col_off = 0;
  o.ldo = N;
  EpiPost e{gelu_col0 < N ? gelu_col0 : INT64_MAX, residual, ld_res, gate, gate_ld, rows_per_gate};
  return launch_gemm_to(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, false, a, w, a_scale,
                        w_scale, bias, o, out_dtype, M, N, K, static_cast<cudaStream_t>(stream), &e);
}

QLIN_API int qlin_gemm_w8a8_fused_segments(const int8_t* a, const float* a_scale, const int8_t* w,
                                           const float* w_scale, int wscale_mode, const void* bias, void* out,
                                           int out_dtype, int64_t M, int64_t N, int64_t K, int64_t gelu_col0,
                                           const void* residual, int64_t ld_res, const void* gate, int64_t gate_ld,
                                           int64_t rows_per_gate, int64_t a_seg_rows, int64_t a_seg_stride,
                                           int64_t a_seg_off, int64_t out_seg_rows, int64_t out_seg_stride,
                                           int64_t out_seg_off, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (out_dtype != QLIN_BF16 && out_dtype != QLIN_F16)
    return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16 or F16 for segmented rows");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  if (gelu_col0 < 0) return fail(QLIN_ERR_INVALID_ARG, "gelu_col0 < 0");
  if (gate && !residual) return fail(QLIN_ERR_INVALID_ARG, "a gate needs a residual");
  if (residual && ld_res < N) return fail(QLIN_ERR_INVALID_ARG, "ld_res < N");
  if (gate && gate_ld < N) return fail(QLIN_ERR_INVALID_ARG, "gate_ld < N");
  if ((residual && (!aligned16(residual) || (ld_res * 2) % 16)) || (gate && (!aligned16(gate) || (gate_ld * 2) % 16)))
    return fail(QLIN_ERR_ALIGNMENT, "residual and gate rows must be 16-byte aligned");
  if (N % 8 || !aligned16(out)) return fail(QLIN_ERR_ALIGNMENT, "segmented output rows need N % 8 == 0, aligned out");
  OutSpec o;
  for (int i = 0; i < 8; ++i) o.outs[i] = nullptr;
  o.outs[0] = out;
  o.nout = 1;
  o.col_off = 0;
  o.ldo = N;
  GemmSegments sg{a_seg_rows, a_seg_stride, a_seg_off, out_seg_rows, out_seg_stride, out_seg_off};
  const bool post = gelu_col0 < N || residual != nullptr;
  EpiPost e{gelu_col0 < N ? gelu_col0 : INT64_MAX, residual, ld_res, gate, gate_ld, rows_per_gate};
  return launch_gemm_to(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, false, a, w, a_scale,
                        w_scale, bias, o, out_dtype, M, N, K, static_cast<cudaStream_t>(stream), post ? &e : nullptr,
                        &sg);
}

QLIN_API int qlin_gemm_w8a8_allgather(const int8_t* a, const float* a_scale, const int8_t* w_shard,
                                      const float* w_scale_shard, int wscale_mode, const void* bias_shard,
                                      void* const* out_bufs, int n_out, int64_t col_off, int64_t ldo, int out_dtype,
                                      int64_t M, int64_t N_shard, int64_t K, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w_shard, M, N_shard, K, 16);
  if (rc || M == 0 || N_shard == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_scale_shard || !out_bufs) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  if (wscale_mode != QLIN_WSCALE_ROW && wscale_mode != QLIN_WSCALE_TENSOR)
    return fail(QLIN_ERR_INVALID_ARG, "bad wscale_mode");
  if (n_out < 1 || n_out > 8) return fail(QLIN_ERR_INVALID_ARG, "n_out must be between 1 and 8");
  if (col_off < 0 || ldo < col_off + N_shard) return fail(QLIN_ERR_INVALID_ARG, "col_off + N_shard > ldo");
  const int es = esize(out_dtype);
  if ((col_off * es) % 16 || (ldo * es) % 16) return fail(QLIN_ERR_ALIGNMENT, "col_off and ldo must be 16-byte aligned");
  OutSpec o;
  o.nout = n_out;
  o.col_off = col_off;
  o.ldo = ldo;
  for (int i = 0; i < 8; ++i) o.outs[i] = nullptr;
  for (int i = 0; i < n_out; ++i) {
    if (!out_bufs[i]) return fail(QLIN_ERR_INVALID_ARG, "null output buffer");
    if (!aligned16(out_bufs[i])) return fail(QLIN_ERR_ALIGNMENT, "output buffers must be 16-byte aligned");
    o.outs[i] = out_bufs[i];
  }
  return launch_gemm_to(wscale_mode == QLIN_WSCALE_ROW ? GEMM_W8A8_ROW : GEMM_W8A8_TENSOR, false, a, w_shard,
                        a_scale, w_scale_shard, bias_shard, o, out_dtype, M, N_shard, K,
                        static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_int_mm(const int8_t* a, const int8_t* w, int32_t* c, int64_t M, int64_t N, int64_t K,
                         void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w, M, N, K, 16);
  if (rc || M == 0 || N == 0) return rc;
  if (!c) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  return launch_gemm(GEMM_I32, false, a, w, nullptr, nullptr, nullptr, c, QLIN_F32, M, N, K,
                     static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_int4_mm(const int8_t* a, const int8_t* w_packed, int32_t* c, int64_t M, int64_t N, int64_t K,
                          void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w_packed, M, N, K, 32);
  if (rc || M == 0 || N == 0) return rc;
  if (!c) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  return launch_gemm(GEMM_I32, true, a, w_packed, nullptr, nullptr, nullptr, c, QLIN_F32, M, N, K,
                     static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w4a4(const int8_t* a, const float* a_scale, const int8_t* w_packed, const float* w_scale,
                            const void* bias, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                            void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w_packed, M, N, K, 32);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  return launch_gemm(GEMM_W4A4_ROW, true, a, w_packed, a_scale, w_scale, bias, out, out_dtype, M, N, K,
                     static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w4a8_g128(const int8_t* a, const float* a_scale, const int8_t* w_packed,
                                 const uint16_t* w_gscale_bf16, const void* bias, void* out, int out_dtype,
                                 int64_t M, int64_t N, int64_t K, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w_packed, M, N, K, 128);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_scale || !w_gscale_bf16 || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  return launch_gemm_g128(false, a, a_scale, w_packed, w_gscale_bf16, bias, out, out_dtype, M, N, K,
                          static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_gemm_w4a4_g128(const int8_t* a, const float* a_gscale, const int8_t* w_packed,
                                 const uint16_t* w_gscale_bf16, const void* bias, void* out, int out_dtype,
                                 int64_t M, int64_t N, int64_t K, void* stream) {
  QLIN_RANGE();
  int rc = gemm_common_checks(a, w_packed, M, N, K, 128);
  if (rc || M == 0 || N == 0) return rc;
  if (!float_dt(out_dtype)) return fail(QLIN_ERR_INVALID_ARG, "out_dtype must be BF16, F16 or F32");
  if (!a_gscale || !w_gscale_bf16 || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  return launch_gemm_g128(true, a, a_gscale, w_packed, w_gscale_bf16, bias, out, out_dtype, M, N, K,
                          static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_weight_int8(const void* w, int w_dtype, int64_t N, int64_t K, int rot_kind, int rot_group,
                                    float rot_c, int8_t* q, float* scale, void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(w_dtype)) return fail(QLIN_ERR_INVALID_ARG, "w_dtype must be BF16, F16 or F32");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!w || !q || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (!rows_vec_ok(w, K, K, w_dtype) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "weights need K % 16 == 0 and 16-byte alignment");
  RowQuantLaunch L{w_dtype, QLIN_F32, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, MODE_INT8};
  return launch_rowquant(L, w, K, N, K, rot_c, 0.0f, nullptr, 0, q, scale, nullptr, 0,
                         static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_quant_weight_int4(const void* w, int w_dtype, int64_t N, int64_t K, int rot_kind, int rot_group,
                                    float rot_c, int group, int8_t* packed, float* scale, void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(w_dtype)) return fail(QLIN_ERR_INVALID_ARG, "w_dtype must be BF16, F16 or F32");
  if (group != 0 && group != 128) return fail(QLIN_ERR_UNSUPPORTED, "int4 group must be 0 or 128");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!w || !packed || !scale) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (!rows_vec_ok(w, K, K, w_dtype) || (K % 32) || !aligned16(packed) || (group && K % 128))
    return fail(QLIN_ERR_ALIGNMENT, "int4 weights need K % 32 == 0 (K % 128 for groups) and 16-byte alignment");
  // group == 0: float32 math (quantize_convrot_w4a4_weight on a .float() weight);
  // group == 128: the compute dtype is the weight dtype.
  const int dt_q = group ? w_dtype : QLIN_F32;
  const float cmin = group ? clamp_min_for(w_dtype) : 1e-10f;
  RowQuantLaunch L{w_dtype, dt_q, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group,
                   group ? MODE_INT4_G128 : MODE_INT4_ROW};
  return launch_rowquant(L, w, K, N, K, rot_c, cmin, nullptr, 0, nullptr, scale, packed, 0,
                         static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_requant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                                    const uint8_t* s_rel_fp8, int group_size, int64_t N, int64_t K, int8_t* q,
                                    float* scale, void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0 || group_size <= 0 || K % group_size)
    return fail(QLIN_ERR_INVALID_ARG, "bad shape / group_size");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!packed || !codebook || !s_channel || !s_rel_fp8 || !q || !scale)
    return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if (K % 32 || !aligned16(packed) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "need K % 32 == 0 and 16-byte alignment");
  return launch_requant_asym_w4a8(packed, codebook, s_channel, s_rel_fp8, group_size, N, K, q, scale, nullptr,
                                  static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_dequant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                                    const uint8_t* s_rel_fp8, int group_size, int64_t N, int64_t K, float* out,
                                    void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0 || group_size <= 0 || K % group_size)
    return fail(QLIN_ERR_INVALID_ARG, "bad shape / group_size");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!packed || !codebook || !s_channel || !s_rel_fp8 || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if (K % 32 || !aligned16(packed) || !aligned16(out))
    return fail(QLIN_ERR_ALIGNMENT, "need K % 32 == 0 and 16-byte alignment");
  return launch_requant_asym_w4a8(packed, codebook, s_channel, s_rel_fp8, group_size, N, K, nullptr, nullptr, out,
                                  static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_dequant_int8(const int8_t* q, const float* scale, int scale_mode, int64_t N, int64_t K,
                               int rot_kind, int rot_group, float rot_c, float* out, void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!q || !scale || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (K % 16 || !aligned16(q) || !aligned16(out))
    return fail(QLIN_ERR_ALIGNMENT, "need K % 16 == 0 and 16-byte alignment");
  RowQuantLaunch L{DT_I8, QLIN_F32, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group, MODE_ROTATE};
  return launch_rowquant(L, q, K, N, K, rot_c, 0.0f, scale, scale_mode == QLIN_WSCALE_ROW, nullptr, nullptr, out, 0,
                         static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_requant_int8(const float* w, const float* scale, int scale_mode, int64_t N, int64_t K,
                               int rot_kind, int rot_group, float rot_c, int round_mode, uint64_t seed, int8_t* q,
                               void* stream) {
  QLIN_RANGE();
  if (N < 0 || K < 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (round_mode != QLIN_ROUND_NEAREST && round_mode != QLIN_ROUND_STOCHASTIC)
    return fail(QLIN_ERR_INVALID_ARG, "bad round_mode");
  if (N == 0 || K == 0) return QLIN_OK;
  if (!w || !scale || !q) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  if ((rc = check_rot(rot_kind, rot_group, K))) return rc;
  if (K % 16 || !aligned16(w) || !aligned16(q))
    return fail(QLIN_ERR_ALIGNMENT, "need K % 16 == 0 and 16-byte alignment");
  RowQuantLaunch L{QLIN_F32, QLIN_F32, rot_kind, rot_kind == QLIN_ROT_NONE ? 0 : rot_group,
                   round_mode == QLIN_ROUND_NEAREST ? MODE_REQUANT : MODE_REQUANT_SR};
  return launch_rowquant(L, w, K, N, K, rot_c, 0.0f, scale, scale_mode == QLIN_WSCALE_ROW, q, nullptr, nullptr, seed,
                         static_cast<cudaStream_t>(stream));
}

QLIN_API int qlin_situ(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, void* out, void* stream) {
  QLIN_RANGE();
  if (M < 0 || K < 0 || ldx < 2 * K) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (!float_dt(x_dtype)) return fail(QLIN_ERR_INVALID_ARG, "x_dtype must be BF16, F16 or F32");
  if (M == 0 || K == 0) return QLIN_OK;
  if (!x || !out) return fail(QLIN_ERR_INVALID_ARG, "null pointer");
  int rc = check_device();
  if (rc) return rc;
  return launch_situ(x_dtype, x, ldx, M, K, out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
