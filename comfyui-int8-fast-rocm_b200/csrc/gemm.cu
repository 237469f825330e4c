// Host side of the tcgen05 GEMMs: TMA descriptors, tile configuration, launch.
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <mutex>

#include "../../include/qlinear_b200.h"
#include "gemm_g128.cuh"
#include "gemm_i8.cuh"
#include "internal.h"

namespace qlin {
namespace {

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t get_encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(ptr);
  });
  return fn;
}

// 2-D tensor map: `outer` rows of `inner` elements, row pitch `pitch` bytes
// (uint8 elements unless `dtype` says otherwise).
int make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t pitch, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapSwizzle swz,
              CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8) {
  PFN_encodeTiled_t enc = get_encode_fn();
  if (!enc) return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ")");
  return QLIN_OK;
}

// 3-D tensor map of segmented rows: `nseg` segments of `seg_rows` rows of
// `inner` elements; rows `pitch` bytes apart within a segment, segments
// `seg_pitch` bytes apart; boxes of box_inner x box_rows x 1.
int make_tmap3(CUtensorMap* m, const void* base, uint64_t inner, uint64_t seg_rows, uint64_t nseg, uint64_t pitch,
               uint64_t seg_pitch, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz,
               CUtensorMapDataType dtype) {
  PFN_encodeTiled_t enc = get_encode_fn();
  if (!enc) return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t dims[3] = {inner, seg_rows, nseg};
  cuuint64_t strides[2] = {pitch, seg_pitch};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(QLIN_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (code " + std::to_string((int)r) + ")");
  return QLIN_OK;
}

// QLIN_NO_NARROW_TAIL=1 keeps every tile of the CTA-pair kernel 256 columns
// wide (comparison runs).
bool narrow_tail_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_NO_NARROW_TAIL");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}

template <int BN, int EPI, int OUT_DT, bool B_INT4>
int launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, B_INT4>;
  auto kern = gemm_i8_kernel<BN, EPI, OUT_DT, B_INT4>;
  static std::atomic<uint64_t> attr_devices{0};  // smem limit raised once per device
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  cudaError_t e;
  if (!(attr_devices.load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm)");
    attr_devices.fetch_or(bit);
  }
  const int num_tiles = ((p.M + GEMM_BM - 1) / GEMM_BM) * ((p.N + BN - 1) / BN);
  const int grid = num_tiles < p.num_sms ? num_tiles : p.num_sms;
  kern<<<grid, Cfg::NUM_THREADS, Cfg::SMEM_BYTES, stream>>>(ta, tb, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return QLIN_OK;
}

template <int EPI, int OUT_DT, bool SPLIT = false, bool B_INT4 = false>
int launch_pair_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, cudaStream_t stream) {
  using Cfg = PairCfg<EPI, OUT_DT, B_INT4>;
  auto kern = gemm_i8_pair_kernel<EPI, OUT_DT, SPLIT, B_INT4>;
  // 16-bit output through TMA stores: one destination, 16-byte aligned rows
  CUtensorMap tc = ta;
  int use_tma_store = 0;
  if (Cfg::TMA_ST && p.nout == 1 && (p.ldo * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
      (p.col_off * 2) % 16 == 0) {
    int rc;
    if (p.o_seg == 0) {
      rc = make_tmap(&tc, p.out, (uint64_t)(p.col_off + p.N), (uint64_t)p.M, (uint64_t)p.ldo * 2, 32, 32,
                     CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_DATA_TYPE_UINT16);
    } else {
      rc = make_tmap3(&tc, static_cast<const uint16_t*>(p.out) + p.o_seg_off * p.ldo, (uint64_t)(p.col_off + p.N),
                      (uint64_t)p.o_seg, (uint64_t)(p.M / p.o_seg), (uint64_t)p.ldo * 2,
                      (uint64_t)p.o_seg_stride * p.ldo * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_DATA_TYPE_UINT16);
    }
    if (rc) return rc;
    use_tma_store = 1;
  }
  if (p.o_seg != 0 && !use_tma_store)
    return fail(QLIN_ERR_UNSUPPORTED, "segmented output rows need a 16-bit, 16-byte aligned single destination");
  static std::atomic<uint64_t> attr_devices{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  cudaError_t e;
  if (!(attr_devices.load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm pair)");
    attr_devices.fetch_or(bit);
  }
  const int num_tiles = ((p.M + 2 * GEMM_BM - 1) / (2 * GEMM_BM)) * ((p.N + Cfg::BN - 1) / Cfg::BN);
  // Narrow last wave (plain 16-bit epilogue through TMA stores, one
  // destination, no split K): when the tiles leave a last wave that fills at
  // most half of the CTA pairs, that wave's tiles run as two 128-column
  // units each.  QLIN_NO_NARROW_TAIL=1 keeps every tile full width.
  GemmParams pn = p;
  const int all_clusters = p.num_sms / 2;
  const int rem = all_clusters > 0 ? num_tiles % all_clusters : 0;
  if (!SPLIT && !B_INT4 && !(EPI & EPI_POST) && EPI != EPI_I32 && use_tma_store && num_tiles > all_clusters &&
      rem > 0 && 2 * rem <= all_clusters && !narrow_tail_disabled())
    pn.narrow_first = num_tiles - rem;
  const int num_units = SPLIT ? num_tiles * p.splits
                              : (pn.narrow_first > 0 ? pn.narrow_first + 2 * (num_tiles - pn.narrow_first) : num_tiles);
  const int clusters = num_units < p.num_sms / 2 ? num_units : p.num_sms / 2;
  e = launch_pdl(kern, dim3(2 * clusters), dim3(Cfg::NUM_THREADS), Cfg::SMEM_BYTES, stream, ta, tb, tc, pn,
                 use_tma_store);
  if (e != cudaSuccess) return cuda_fail(e, "gemm pair launch");
  return QLIN_OK;
}

int dispatch_pair(int kind, int out_dt, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                  cudaStream_t s, bool post = false) {
  if (post) {  // 16-bit outputs only (checked by the caller)
    if (kind == GEMM_W8A8_ROW) {
      if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_ROW | EPI_POST, DT_BF16>(ta, tb, p, s);
      if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_ROW | EPI_POST, DT_F16>(ta, tb, p, s);
    }
    if (kind == GEMM_W8A8_TENSOR) {
      if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_TENSOR | EPI_POST, DT_BF16>(ta, tb, p, s);
      if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_TENSOR | EPI_POST, DT_F16>(ta, tb, p, s);
    }
    return fail(QLIN_ERR_UNSUPPORTED, "epilogue steps need a W8A8 GEMM with bf16 or f16 output");
  }
  if (kind == GEMM_I32) return launch_pair_cfg<EPI_I32, DT_F32>(ta, tb, p, s);
  if (kind == GEMM_W8A8_ROW) {
    if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_ROW, DT_BF16>(ta, tb, p, s);
    if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_ROW, DT_F16>(ta, tb, p, s);
    if (out_dt == DT_F32) return launch_pair_cfg<EPI_W8A8_ROW, DT_F32>(ta, tb, p, s);
  }
  if (kind == GEMM_W8A8_TENSOR) {
    if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_BF16>(ta, tb, p, s);
    if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_F16>(ta, tb, p, s);
    if (out_dt == DT_F32) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_F32>(ta, tb, p, s);
  }
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported GEMM epilogue / output dtype");
}

template <int BN, bool B_INT4>
int dispatch_epi(int kind, int out_dt, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                 cudaStream_t s, bool post = false) {
  if constexpr (!B_INT4) {
    if (post) {
      if (kind == GEMM_W8A8_ROW) {
        if (out_dt == DT_BF16) return launch_cfg<BN, EPI_W8A8_ROW | EPI_POST, DT_BF16, false>(ta, tb, p, s);
        if (out_dt == DT_F16) return launch_cfg<BN, EPI_W8A8_ROW | EPI_POST, DT_F16, false>(ta, tb, p, s);
      }
      if (kind == GEMM_W8A8_TENSOR) {
        if (out_dt == DT_BF16) return launch_cfg<BN, EPI_W8A8_TENSOR | EPI_POST, DT_BF16, false>(ta, tb, p, s);
        if (out_dt == DT_F16) return launch_cfg<BN, EPI_W8A8_TENSOR | EPI_POST, DT_F16, false>(ta, tb, p, s);
      }
      return fail(QLIN_ERR_UNSUPPORTED, "epilogue steps need a W8A8 GEMM with bf16 or f16 output");
    }
  } else {
    if (post) return fail(QLIN_ERR_UNSUPPORTED, "epilogue steps need a W8A8 GEMM with bf16 or f16 output");
  }
  if (kind == GEMM_I32) return launch_cfg<BN, EPI_I32, DT_F32, B_INT4>(ta, tb, p, s);
  if constexpr (!B_INT4) {
    if (kind == GEMM_W8A8_ROW) {
      if (out_dt == DT_BF16) return launch_cfg<BN, EPI_W8A8_ROW, DT_BF16, false>(ta, tb, p, s);
      if (out_dt == DT_F16) return launch_cfg<BN, EPI_W8A8_ROW, DT_F16, false>(ta, tb, p, s);
      if (out_dt == DT_F32) return launch_cfg<BN, EPI_W8A8_ROW, DT_F32, false>(ta, tb, p, s);
    }
    if (kind == GEMM_W8A8_TENSOR) {
      if (out_dt == DT_BF16) return launch_cfg<BN, EPI_W8A8_TENSOR, DT_BF16, false>(ta, tb, p, s);
      if (out_dt == DT_F16) return launch_cfg<BN, EPI_W8A8_TENSOR, DT_F16, false>(ta, tb, p, s);
      if (out_dt == DT_F32) return launch_cfg<BN, EPI_W8A8_TENSOR, DT_F32, false>(ta, tb, p, s);
    }
  } else {
    if (kind == GEMM_W4A4_ROW) {
      if (out_dt == DT_BF16) return launch_cfg<BN, EPI_W4A4_ROW, DT_BF16, true>(ta, tb, p, s);
      if (out_dt == DT_F16) return launch_cfg<BN, EPI_W4A4_ROW, DT_F16, true>(ta, tb, p, s);
      if (out_dt == DT_F32) return launch_cfg<BN, EPI_W4A4_ROW, DT_F32, true>(ta, tb, p, s);
    }
  }
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported GEMM epilogue / output dtype");
}

// QLIN_GEMM_NO_PAIR=1 forces the single-CTA kernel (comparison runs).
bool pair_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_GEMM_NO_PAIR");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}

// QLIN_INT4_NO_PAIR=1 keeps packed-int4 GEMMs on the single-CTA kernel
// (comparison runs).
bool int4_pair_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_INT4_NO_PAIR");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}

GemmParams make_params(int64_t M, int64_t N, int64_t K, const float* a_scale, const float* w_scale, const void* bias,
                       const OutSpec& o, int sms) {
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_scale = a_scale;
  p.w_scale = w_scale;
  p.bias = bias;
  p.out = o.outs[0];
  p.ldo = o.ldo;
  p.num_sms = sms;
  p.nout = o.nout;
  p.col_off = o.col_off;
  for (int i = 0; i < kMaxOutputs; ++i) p.outs[i] = i < o.nout ? o.outs[i] : nullptr;
  p.gelu_col0 = INT64_MAX;  // EPI_POST fields: no GELU, no residual
  p.rows_per_gate = 1;
  p.stall_kb = -1;
  p.splits = 1;
  p.kb_split = (int)((K + GEMM_BK - 1) / GEMM_BK);
  return p;
}

void set_post(GemmParams& p, const EpiPost& e) {
  p.gelu_col0 = e.gelu_col0;
  p.residual = e.residual;
  p.ld_res = e.ld_res;
  p.gate = e.gate;
  p.gate_ld = e.gate_ld;
  p.rows_per_gate = e.rows_per_gate > 0 ? e.rows_per_gate : INT64_MAX;
}

}  // namespace

int launch_gemm(int kind, bool b_int4, const int8_t* a, const int8_t* b, const float* a_scale,
                const float* w_scale, const void* bias, void* out, int out_dt, int64_t M, int64_t N, int64_t K,
                cudaStream_t stream) {
  OutSpec o;
  o.outs[0] = out;
  o.nout = 1;
  o.col_off = 0;
  o.ldo = N;
  return launch_gemm_to(kind, b_int4, a, b, a_scale, w_scale, bias, o, out_dt, M, N, K, stream);
}

int launch_gemm_to(int kind, bool b_int4, const int8_t* a, const int8_t* b, const float* a_scale,
                   const float* w_scale, const void* bias, const OutSpec& o, int out_dt, int64_t M, int64_t N,
                   int64_t K, cudaStream_t stream, const EpiPost* post, const GemmSegments* seg) {
  if (M == 0 || N == 0) return QLIN_OK;
  if (o.nout < 1 || o.nout > kMaxOutputs) return fail(QLIN_ERR_INVALID_ARG, "between 1 and 8 outputs");
  if (post != nullptr && o.nout != 1) return fail(QLIN_ERR_UNSUPPORTED, "epilogue steps need one destination");
  const int sms = device_sm_count();
  if (sms <= 0) return fail(QLIN_ERR_NO_DEVICE, "no CUDA device");
  const bool segmented = seg != nullptr && (seg->a_rows != 0 || seg->o_rows != 0);
  if (segmented) {
    if (b_int4 || (kind != GEMM_W8A8_ROW && kind != GEMM_W8A8_TENSOR) || o.nout != 1 ||
        (out_dt != DT_BF16 && out_dt != DT_F16) || M < 256 || N < 256 || sms < 2 || pair_disabled())
      return fail(QLIN_ERR_UNSUPPORTED, "segmented rows: W8A8 on CTA pairs with a 16-bit output, M and N >= 256");
    if (seg->a_rows < 0 || seg->o_rows < 0 || seg->a_rows % 128 != 0 || seg->o_rows % 32 != 0 ||
        (seg->a_rows && (M % seg->a_rows != 0 || seg->a_stride < seg->a_rows || seg->a_off < 0 ||
                         seg->a_off + seg->a_rows > seg->a_stride)) ||
        (seg->o_rows && (M % seg->o_rows != 0 || seg->o_stride < seg->o_rows || seg->o_off < 0 ||
                         seg->o_off + seg->o_rows > seg->o_stride)) ||
        seg->a_rows > INT32_MAX || seg->o_rows > INT32_MAX)
      return fail(QLIN_ERR_INVALID_ARG,
                  "segments: rows a multiple of 128 (A) / 32 (output) dividing M, inside a stride >= offset + rows");
  }
  CUtensorMap ta, tb;
  // Large int8 x int8 problems run on CTA pairs (256 x 256 tiles).
  if (!b_int4 && kind != GEMM_W4A4_ROW && M >= 256 && N >= 256 && sms >= 2 && !pair_disabled()) {
    int rc;
    if (segmented && seg->a_rows) {
      rc = make_tmap3(&ta, a + seg->a_off * K, (uint64_t)K, (uint64_t)seg->a_rows, (uint64_t)(M / seg->a_rows),
                      (uint64_t)K, (uint64_t)(seg->a_stride * K), GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_DATA_TYPE_UINT8);
    } else {
      rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
    rc = make_tmap(&tb, b, (uint64_t)K, (uint64_t)N, (uint64_t)K, GEMM_BK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    GemmParams p = make_params(M, N, K, a_scale, w_scale, bias, o, sms);
    if (post != nullptr) set_post(p, *post);
    if (segmented) {
      p.a_seg = (int)seg->a_rows;
      p.a_seg_stride = seg->a_stride;
      p.a_seg_off = seg->a_off;
      p.o_seg = (int)seg->o_rows;
      p.o_seg_stride = seg->o_stride;
      p.o_seg_off = seg->o_off;
    }
    return dispatch_pair(kind, out_dt, ta, tb, p, stream, post != nullptr);
  }
  if (segmented) return fail(QLIN_ERR_UNSUPPORTED, "segmented rows need the CTA-pair kernel");
  // Packed-int4 weights on CTA pairs (each CTA unpacks its own 128 rows).
  if (b_int4 && (kind == GEMM_W4A4_ROW || kind == GEMM_I32) && post == nullptr && o.nout == 1 && M >= 256 &&
      N >= 256 && sms >= 2 && !pair_disabled() && !int4_pair_disabled()) {
    int rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap(&tb, b, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), GEMM_BK / 2, 128,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    GemmParams p = make_params(M, N, K, a_scale, w_scale, bias, o, sms);
    if (kind == GEMM_I32) return launch_pair_cfg<EPI_I32, DT_F32, false, true>(ta, tb, p, stream);
    if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W4A4_ROW, DT_BF16, false, true>(ta, tb, p, stream);
    if (out_dt == DT_F16) return launch_pair_cfg<EPI_W4A4_ROW, DT_F16, false, true>(ta, tb, p, stream);
    if (out_dt == DT_F32) return launch_pair_cfg<EPI_W4A4_ROW, DT_F32, false, true>(ta, tb, p, stream);
    return fail(QLIN_ERR_UNSUPPORTED, "unsupported W4A4 output dtype");
  }
  // Narrow outputs waste half a 256-wide tile; use 128 columns there.
  const int BN = (N <= 128) ? 128 : 256;
  int rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (b_int4) {
    rc = make_tmap(&tb, b, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), GEMM_BK / 2, (uint32_t)BN,
                   CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    rc = make_tmap(&tb, b, (uint64_t)K, (uint64_t)N, (uint64_t)K, GEMM_BK, (uint32_t)BN, CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  GemmParams p = make_params(M, N, K, a_scale, w_scale, bias, o, sms);
  if (post != nullptr) set_post(p, *post);
  const bool ps = post != nullptr;
  if (b_int4) {
    if (BN == 128) return dispatch_epi<128, true>(kind, out_dt, ta, tb, p, stream, ps);
    return dispatch_epi<256, true>(kind, out_dt, ta, tb, p, stream, ps);
  }
  if (BN == 128) return dispatch_epi<128, false>(kind, out_dt, ta, tb, p, stream, ps);
  return dispatch_epi<256, false>(kind, out_dt, ta, tb, p, stream, ps);
}

namespace {

// QLIN_G128_NO_PAIR=1 forces the single-CTA group-128 kernel (comparison runs).
bool g128_pair_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_G128_NO_PAIR");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}

template <int MODE, int OUT_DT>
int launch_g128_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const G128Params& p, int sms, cudaStream_t stream) {
  auto kern = gemm_g128_kernel<MODE, OUT_DT>;
  static std::atomic<uint64_t> attr_devices{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  cudaError_t e;
  if (!(attr_devices.load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G128Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm g128)");
    attr_devices.fetch_or(bit);
  }
  const int num_tiles = ((p.M + G128Cfg::BM - 1) / G128Cfg::BM) * ((p.N + G128Cfg::BN - 1) / G128Cfg::BN);
  const int grid = num_tiles < sms ? num_tiles : sms;
  kern<<<grid, G128Cfg::NUM_THREADS, G128Cfg::SMEM_BYTES, stream>>>(ta, tb, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm g128 launch");
  return QLIN_OK;
}

template <int MODE, int OUT_DT>
int launch_g128_pair_cfg(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const G128Params& p,
                         int sms, cudaStream_t stream) {
  auto kern = gemm_g128_pair_kernel<MODE, OUT_DT>;
  static std::atomic<uint64_t> attr_devices{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);
  cudaError_t e;
  if (!(attr_devices.load() & bit)) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G128PairCfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm g128 pair)");
    attr_devices.fetch_or(bit);
  }
  const int num_tiles = ((p.M + 2 * G128PairCfg::BM - 1) / (2 * G128PairCfg::BM)) *
                        ((p.N + G128PairCfg::BN - 1) / G128PairCfg::BN);
  const int clusters = num_tiles < sms / 2 ? num_tiles : sms / 2;
  kern<<<2 * clusters, G128PairCfg::NUM_THREADS, G128PairCfg::SMEM_BYTES, stream>>>(ta, tb, tc, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm g128 pair launch");
  return QLIN_OK;
}

template <int MODE>
int dispatch_g128(int out_dt, const CUtensorMap& ta, const CUtensorMap& tb, const int8_t* w_packed,
                  const G128Params& p, int sms, cudaStream_t s) {
  // 16-bit outputs with 16-byte aligned rows and K a multiple of two scale
  // groups: the CTA-pair kernel (TMA-store epilogue, two groups per step)
  if ((out_dt == DT_BF16 || out_dt == DT_F16) && (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 &&
      (p.ldo * 2) % 16 == 0 && p.K % G128PairCfg::KS == 0 && !g128_pair_disabled()) {
    CUtensorMap tc, tb2;  // the pair loads 64 packed weight rows of a two-group step per CTA
    int rc = make_tmap(&tc, p.out, (uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.ldo * 2, 32, 32,
                       CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_DATA_TYPE_UINT16);
    if (rc) return rc;
    rc = make_tmap(&tb2, w_packed, (uint64_t)(p.K / 2), (uint64_t)p.N, (uint64_t)(p.K / 2), G128PairCfg::KS / 2,
                   G128PairCfg::BNH, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    if (out_dt == DT_BF16) return launch_g128_pair_cfg<MODE, DT_BF16>(ta, tb2, tc, p, sms, s);
    return launch_g128_pair_cfg<MODE, DT_F16>(ta, tb2, tc, p, sms, s);
  }
  if (out_dt == DT_BF16) return launch_g128_cfg<MODE, DT_BF16>(ta, tb, p, sms, s);
  if (out_dt == DT_F16) return launch_g128_cfg<MODE, DT_F16>(ta, tb, p, sms, s);
  if (out_dt == DT_F32) return launch_g128_cfg<MODE, DT_F32>(ta, tb, p, sms, s);
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported output dtype");
}

}  // namespace

// Split K for the CTA-pair W8A8 kernel.  A problem whose 256 x 256 tiles
// leave most CTA pairs idle is cut into `splits` (2 or 3) K ranges per tile,
// all running in one wave.  The parts meet through int32 partials in global
// scratch (256 KB per tile and part), so a split costs partial traffic and a
// serialised fix-up: measured on B200, 13-16 us at 48 tiles (1024 x 3072 x
// 3072: 30.8 us split against 20.5 us unsplit), which is why only problems
// with at most one wave of split units and K >= 8192 (64 K-slabs) split.
bool splitk_plan(int64_t M, int64_t N, int64_t K, int sms, int* splits, int* kb_split) {
  *splits = 1;
  *kb_split = (int)((K + GEMM_BK - 1) / GEMM_BK);
  if (M < 256 || N < 256 || sms < 2 || pair_disabled()) return false;
  const int64_t tiles = ((M + 255) / 256) * ((N + 255) / 256);
  if (tiles > SPLITK_MAX_TILES) return false;
  const int64_t clusters = sms / 2;
  const int64_t kb = *kb_split;
  if (kb < 64) return false;
  for (int s = SPLITK_MAX; s >= 2; --s) {
    if (tiles * s > clusters) continue;
    const int64_t per = (kb + s - 1) / s;
    *splits = (int)((kb + per - 1) / per);
    *kb_split = (int)per;
    return *splits > 1;
  }
  return false;
}

size_t splitk_header_bytes() { return SPLITK_HEADER; }

size_t splitk_scratch_bytes(int64_t M, int64_t N, int64_t K) {
  int splits, kb_split;
  if (!splitk_plan(M, N, K, device_sm_count(), &splits, &kb_split)) return 0;
  const int tiles = (int)(((M + 255) / 256) * ((N + 255) / 256));
  return splitk_layout(tiles, splits).bytes;
}

int launch_gemm_splitk(int kind, const int8_t* a, const int8_t* b, const float* a_scale, const float* w_scale,
                       const void* bias, void* out, int out_dt, int64_t M, int64_t N, int64_t K, void* scratch,
                       size_t scratch_bytes, cudaStream_t stream) {
  if (M == 0 || N == 0) return QLIN_OK;
  const int sms = device_sm_count();
  if (sms <= 0) return fail(QLIN_ERR_NO_DEVICE, "no CUDA device");
  int splits, kb_split;
  if (kind == GEMM_I32 || !splitk_plan(M, N, K, sms, &splits, &kb_split))
    return launch_gemm(kind, false, a, b, a_scale, w_scale, bias, out, out_dt, M, N, K, stream);
  const int tiles = (int)(((M + 255) / 256) * ((N + 255) / 256));
  const SplitKLayout l = splitk_layout(tiles, splits);
  if (scratch == nullptr || scratch_bytes < l.bytes)
    return fail(QLIN_ERR_INVALID_ARG, "split-K scratch smaller than qlin_gemm_w8a8_splitk_scratch reports");
  if ((reinterpret_cast<uintptr_t>(scratch) & 255) != 0) return fail(QLIN_ERR_ALIGNMENT, "split-K scratch must be 256-byte aligned");
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap(&tb, b, (uint64_t)K, (uint64_t)N, (uint64_t)K, GEMM_BK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  OutSpec o;
  o.outs[0] = out;
  o.nout = 1;
  o.col_off = 0;
  o.ldo = N;
  GemmParams p = make_params(M, N, K, a_scale, w_scale, bias, o, sms);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  p.splits = splits;
  p.kb_split = kb_split;
  p.sk_count = reinterpret_cast<uint32_t*>(base + l.count_off);
  p.sk_ready = reinterpret_cast<uint32_t*>(base + l.ready_off);
  p.sk_part = reinterpret_cast<int32_t*>(base + l.part_off);
  if (kind == GEMM_W8A8_ROW) {
    if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_ROW, DT_BF16, true>(ta, tb, p, stream);
    if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_ROW, DT_F16, true>(ta, tb, p, stream);
    if (out_dt == DT_F32) return launch_pair_cfg<EPI_W8A8_ROW, DT_F32, true>(ta, tb, p, stream);
  }
  if (kind == GEMM_W8A8_TENSOR) {
    if (out_dt == DT_BF16) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_BF16, true>(ta, tb, p, stream);
    if (out_dt == DT_F16) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_F16, true>(ta, tb, p, stream);
    if (out_dt == DT_F32) return launch_pair_cfg<EPI_W8A8_TENSOR, DT_F32, true>(ta, tb, p, stream);
  }
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported split-K epilogue / output dtype");
}

int launch_gemm_g128(bool a_int4_groups, const int8_t* a, const float* a_scale, const int8_t* w_packed,
                     const uint16_t* w_gscale, const void* bias, void* out, int out_dt, int64_t M, int64_t N,
                     int64_t K, cudaStream_t stream) {
  if (M == 0 || N == 0) return QLIN_OK;
  const int sms = device_sm_count();
  if (sms <= 0) return fail(QLIN_ERR_NO_DEVICE, "no CUDA device");
  if (K % G128Cfg::BK) return fail(QLIN_ERR_ALIGNMENT, "K must be a multiple of 128");
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, G128Cfg::BK, G128Cfg::BM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap(&tb, w_packed, (uint64_t)(K / 2), (uint64_t)N, (uint64_t)(K / 2), G128Cfg::BK / 2, G128Cfg::BN,
                 CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  G128Params p;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.a_scale = a_scale;
  p.w_gscale = w_gscale;
  p.bias = bias;
  p.out = out;
  p.ldo = N;
  if (a_int4_groups) return dispatch_g128<G128_W4A4>(out_dt, ta, tb, w_packed, p, sms, stream);
  return dispatch_g128<G128_W4A8>(out_dt, ta, tb, w_packed, p, sms, stream);
}

namespace {

// One thread waits, bounded, on an mbarrier phase that nothing completes.
__global__ void wait_selftest_kernel() {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait_bounded(&bar, 0, &abort_flag);
}

}  // namespace

int launch_wait_selftest(cudaStream_t stream) {
  wait_selftest_kernel<<<1, 32, 0, stream>>>();
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QLIN_OK : cuda_fail(e, "wait self-test launch");
}

int launch_gemm_stall(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale, void* out,
                      int64_t M, int64_t N, int64_t K, int64_t stall_kb, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return fail(QLIN_ERR_INVALID_ARG, "bad shape");
  if (stall_kb < 0 || stall_kb >= (K + GEMM_BK - 1) / GEMM_BK) return fail(QLIN_ERR_INVALID_ARG, "stall_kb out of range");
  const int sms = device_sm_count();
  if (sms <= 0) return fail(QLIN_ERR_NO_DEVICE, "no CUDA device");
  OutSpec o;
  o.outs[0] = out;
  o.nout = 1;
  o.col_off = 0;
  o.ldo = N;
  GemmParams p = make_params(M, N, K, a_scale, w_scale, nullptr, o, sms);
  p.stall_kb = (int)stall_kb;
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, a, (uint64_t)K, (uint64_t)M, (uint64_t)K, GEMM_BK, GEMM_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (M >= 256 && N >= 256 && sms >= 2) {
    rc = make_tmap(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, GEMM_BK, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    return launch_pair_cfg<EPI_W8A8_ROW, DT_BF16>(ta, tb, p, stream);
  }
  rc = make_tmap(&tb, w, (uint64_t)K, (uint64_t)N, (uint64_t)K, GEMM_BK, 256, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return launch_cfg<256, EPI_W8A8_ROW, DT_BF16, false>(ta, tb, p, stream);
}

int set_gemm_wait_limit(uint64_t ns) {
  const cudaError_t e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
  return e == cudaSuccess ? QLIN_OK : cuda_fail(e, "set wait limit");
}

int read_device_error(cudaStream_t stream, uint32_t* bits) {
  uint32_t h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_error_bits, sizeof(uint32_t), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return cuda_fail(e, "read error word");
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "sync");
  const uint32_t zero = 0;
  e = cudaMemcpyToSymbolAsync(g_error_bits, &zero, sizeof(uint32_t), 0, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return cuda_fail(e, "clear error word");
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "sync");
  *bits = h;
  return QLIN_OK;
}

}  // namespace qlin
