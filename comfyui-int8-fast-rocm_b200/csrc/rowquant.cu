// Instantiation and launch of the row-wise rotate/quantise kernel family.
#include <atomic>
#include <cstdlib>

#include "../../include/qlinear_b200.h"
#include "internal.h"
#include "rowquant.cuh"
#include "rowstrip.cuh"

namespace qlin {
namespace {

// Rotation shapes this build instantiates: none, regular 16/64/256,
// Sylvester 32/128 (the sizes that are not powers of 4).
enum RotCode { RC_NONE, RC_REG16, RC_REG64, RC_REG256, RC_SYL32, RC_SYL128, RC_BAD };

RotCode rot_code(int kind, int group) {
  if (kind == ROT_NONE) return RC_NONE;
  if (kind == ROT_REGULAR) {
    if (group == 16) return RC_REG16;
    if (group == 64) return RC_REG64;
    if (group == 256) return RC_REG256;
  }
  if (kind == ROT_SYLVESTER) {
    if (group == 32) return RC_SYL32;
    if (group == 128) return RC_SYL128;
  }
  return RC_BAD;
}

struct LaunchShape {
  int chunks, tpr, rpc;
  size_t smem;
};

template <int DT_IN, int DT_Q, int KIND, int R, int CHUNKS, int MODE>
int launch_one(const RowQuantParams& p, const LaunchShape& s, cudaStream_t stream) {
  auto kern = rowquant_kernel<DT_IN, DT_Q, KIND, R, CHUNKS, MODE>;
  // Staged kernels can exceed the default 48 KB once the static reduction
  // array is added; raise the limit once per device for this instantiation.
  static std::atomic<uint64_t> attr_devices{0};
  if (s.smem > 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_devices.load() & bit)) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rowquant)");
      attr_devices.fetch_or(bit);
    }
  }
  // Persistent grid: as many CTAs as fit on the device at once (each walks
  // several rows), never more than there are row groups.
  static std::atomic<int> occ_key{-1}, occ_val{1};
  const int key = s.tpr * s.rpc * 4 + (int)(s.smem >> 10);
  int per_sm = occ_val.load();
  if (occ_key.load() != key) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, s.tpr * s.rpc, s.smem);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy query");
    per_sm = nb > 0 ? nb : 1;
    occ_val.store(per_sm);
    occ_key.store(key);
  }
  const int64_t groups = (p.M + s.rpc - 1) / s.rpc;
  const int64_t cap = (int64_t)device_sm_count() * per_sm;
  dim3 block(s.tpr, s.rpc);
  dim3 grid((unsigned)(groups < cap ? groups : cap));
  kern<<<grid, block, s.smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rowquant launch");
  return QLIN_OK;
}

template <int DT_IN, int DT_Q, int KIND, int R, int MODE>
int by_chunks(const RowQuantParams& p, const LaunchShape& s, cudaStream_t stream) {
  if (s.chunks == 1) return launch_one<DT_IN, DT_Q, KIND, R, 1, MODE>(p, s, stream);
  if constexpr (DT_IN == DT_Q) {
    if (s.chunks == 2) return launch_one<DT_IN, DT_Q, KIND, R, 2, MODE>(p, s, stream);
  }
  return fail(QLIN_ERR_UNSUPPORTED, "row length too large for this kernel configuration");
}

template <int DT_IN, int DT_Q, int MODE>
int by_rot(RotCode rc, const RowQuantParams& p, const LaunchShape& s, cudaStream_t stream) {
  switch (rc) {
    case RC_NONE: return by_chunks<DT_IN, DT_Q, ROT_NONE, 1, MODE>(p, s, stream);
    case RC_REG16: return by_chunks<DT_IN, DT_Q, ROT_REGULAR, 1, MODE>(p, s, stream);
    case RC_REG64: return by_chunks<DT_IN, DT_Q, ROT_REGULAR, 4, MODE>(p, s, stream);
    case RC_REG256: return by_chunks<DT_IN, DT_Q, ROT_REGULAR, 16, MODE>(p, s, stream);
    case RC_SYL32: return by_chunks<DT_IN, DT_Q, ROT_SYLVESTER, 2, MODE>(p, s, stream);
    case RC_SYL128: return by_chunks<DT_IN, DT_Q, ROT_SYLVESTER, 8, MODE>(p, s, stream);
    default: return fail(QLIN_ERR_UNSUPPORTED, "unsupported rotation");
  }
}

template <int DT_IN, int DT_Q>
int by_mode(int mode, RotCode rc, const RowQuantParams& p, const LaunchShape& s, cudaStream_t stream) {
  if constexpr (DT_IN == DT_Q) {
    // activation modes (the compute dtype is the input dtype)
    switch (mode) {
      case MODE_INT8: return by_rot<DT_IN, DT_Q, MODE_INT8>(rc, p, s, stream);
      case MODE_INT4_ROW: return by_rot<DT_IN, DT_Q, MODE_INT4_ROW>(rc, p, s, stream);
      case MODE_INT4_G128: return by_rot<DT_IN, DT_Q, MODE_INT4_G128>(rc, p, s, stream);
      case MODE_ROTATE: return by_rot<DT_IN, DT_Q, MODE_ROTATE>(rc, p, s, stream);
      default: break;
    }
    if constexpr (DT_Q == DT_F32) {
      if (mode == MODE_REQUANT) return by_rot<DT_IN, DT_Q, MODE_REQUANT>(rc, p, s, stream);
      if (mode == MODE_REQUANT_SR) return by_rot<DT_IN, DT_Q, MODE_REQUANT_SR>(rc, p, s, stream);
    }
  } else if constexpr (DT_IN == DT_I8) {
    if (mode == MODE_ROTATE) return by_rot<DT_IN, DT_Q, MODE_ROTATE>(rc, p, s, stream);
  } else {
    // weights held in bf16/f16, computed in float32 (w.float() first)
    if (mode == MODE_INT8) return by_rot<DT_IN, DT_Q, MODE_INT8>(rc, p, s, stream);
    if (mode == MODE_INT4_ROW) return by_rot<DT_IN, DT_Q, MODE_INT4_ROW>(rc, p, s, stream);
  }
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported dtype/mode combination");
}

// Activation int8 quantisation (rowquant_x2_kernel): rows stream through a
// shared-memory ring filled by bulk copies.  Returns QLIN_ERR_UNSUPPORTED
// (without launching) when two ring slots do not fit in shared memory; the
// caller then uses the register-prefetch kernel.
constexpr size_t kX2SmemBudget = 200 * 1024;  // hard limit (one CTA)
// Ring target: four or five CTAs per SM for 3072-element bf16 rows.  The
// ring gives up depth for CTAs, so the bytes in flight per SM stay about
// the same.  Measured against a 72 KB target (three CTAs per SM): 16384 x
// 3072 Sylvester-128 in 52 vs 56 us; 4096 x 3072 and 8192 x 12288 unchanged.
constexpr size_t kX2SmemTarget = 48 * 1024;

template <int DT, int KIND, int R, int CHUNKS, bool FUSED>
int launch_x2(const RowQuantParams& p, int nchunks, cudaStream_t stream) {
  auto kern = rowquant_x2_kernel<DT, KIND, R, CHUNKS, FUSED>;
  constexpr int EB = DT == DT_F32 ? 4 : 2;
  const int per = (nchunks + CHUNKS - 1) / CHUNKS;
  const int tpr = ((per + 31) / 32) * 32;
  int rpc = 256 / tpr;
  if (rpc < 1) rpc = 1;
  if (rpc > 32) rpc = 32;
  const size_t row_bytes = (size_t)p.K * EB * (FUSED && p.situ ? 2 : 1);  // source bytes per ring row
  const int slot_bytes = (int)(((size_t)rpc * row_bytes + 127) / 128 * 128);
  const size_t tbuf = (KIND != ROT_NONE && R > 1) ? (size_t)(rpc * tpr / 32) * 512 * sizeof(float) : 0;
  int stages = 4;
  while (stages > 2 && (size_t)stages * slot_bytes + tbuf + stages * 8 > kX2SmemTarget) --stages;
  const size_t smem = (size_t)stages * slot_bytes + tbuf + stages * 8;
  if (smem > kX2SmemBudget) return QLIN_ERR_UNSUPPORTED;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr_devices{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_devices.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kX2SmemBudget);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rowquant x2)");
    attr_devices.fetch_or(bit);
  }
  static std::atomic<int64_t> occ_key{-1};
  static std::atomic<int> occ_val{1};
  const int64_t key = ((int64_t)tpr * rpc << 32) | (int64_t)smem;
  int per_sm = occ_val.load();
  if (occ_key.load() != key) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, tpr * rpc, smem);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy query");
    per_sm = nb > 0 ? nb : 1;
    occ_val.store(per_sm);
    occ_key.store(key);
  }
  const int64_t groups = (p.M + rpc - 1) / rpc;
  const int64_t cap = (int64_t)device_sm_count() * per_sm;
  cudaError_t e = launch_pdl(kern, dim3((unsigned)(groups < cap ? groups : cap)), dim3(tpr, rpc), smem, stream, p,
                             stages, slot_bytes);
  if (e != cudaSuccess) return cuda_fail(e, "rowquant x2 launch");
  return QLIN_OK;
}

template <int DT, int CHUNKS, bool FUSED>
int x2_by_rot(RotCode rc, const RowQuantParams& p, int nchunks, cudaStream_t s) {
  switch (rc) {
    case RC_NONE: return launch_x2<DT, ROT_NONE, 1, CHUNKS, FUSED>(p, nchunks, s);
    case RC_REG16: return launch_x2<DT, ROT_REGULAR, 1, CHUNKS, FUSED>(p, nchunks, s);
    case RC_REG64: return launch_x2<DT, ROT_REGULAR, 4, CHUNKS, FUSED>(p, nchunks, s);
    case RC_REG256: return launch_x2<DT, ROT_REGULAR, 16, CHUNKS, FUSED>(p, nchunks, s);
    case RC_SYL32: return launch_x2<DT, ROT_SYLVESTER, 2, CHUNKS, FUSED>(p, nchunks, s);
    case RC_SYL128: return launch_x2<DT, ROT_SYLVESTER, 8, CHUNKS, FUSED>(p, nchunks, s);
    default: return fail(QLIN_ERR_UNSUPPORTED, "unsupported rotation");
  }
}

// Chunks per thread: per-row work is amortised over more elements for long
// rows, while short rows keep a full warp per row.
template <int DT, bool FUSED = false>
int x2_by_chunks(RotCode rc, const RowQuantParams& p, int nchunks, cudaStream_t s) {
  if constexpr (DT != DT_F32) {  // float32 rows would need twice the prefetch registers
    if (nchunks >= 512) return x2_by_rot<DT, 4, FUSED>(rc, p, nchunks, s);
  }
  if (nchunks >= 64) return x2_by_rot<DT, 2, FUSED>(rc, p, nchunks, s);
  return x2_by_rot<DT, 1, FUSED>(rc, p, nchunks, s);
}

// One 128-element strip per thread (rowstrip.cuh): 16-bit activations, K a
// multiple of 128 up to 16384, rows 16-byte aligned, codes 32-byte aligned.
template <int DT, int KIND, int G, int SW = STRIP>
int launch_strip(const RowQuantParams& p, cudaStream_t stream) {
  auto kern = rowquant_strip_kernel<DT, KIND, G, SW>;
  const int T = p.K / SW;
  int rows = 128 / T;  // whole rows per CTA; prefer whole warps
  for (int r = rows; r >= 1; --r)
    if ((r * T) % 32 == 0) { rows = r; break; }
  const int threads = rows * T;
  const int slot_bytes = (rows * p.K * 2 + 127) / 128 * 128;
  constexpr int stages = 2;  // measured: 3 or 4 slots were no faster (fewer CTAs per SM)
  const size_t smem = (size_t)stages * slot_bytes;
  if (smem > 200 * 1024) return QLIN_ERR_UNSUPPORTED;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<uint64_t> attr_devices{0};
  const uint64_t bit = 1ull << (dev & 63);
  if (!(attr_devices.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(rowquant strip)");
    attr_devices.fetch_or(bit);
  }
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess) return cuda_fail(e, "occupancy query");
  if (per_sm < 1) per_sm = 1;
  const int64_t nblocks = ((int64_t)p.M + rows - 1) / rows;
  const int64_t cap = (int64_t)device_sm_count() * per_sm;
  e = launch_pdl(kern, dim3((unsigned)(nblocks < cap ? nblocks : cap)), dim3(threads), smem, stream, p.x, p.ldx, p.x2,
                 p.ldx2, p.k1, p.M, p.K, rows, stages, slot_bytes, p.rot_c, p.one, p.q, p.scale);
  if (e != cudaSuccess) return cuda_fail(e, "rowquant strip launch");
  return QLIN_OK;
}

// The strip kernel serves the Sylvester-128 rotation, whose 128-element group
// is one strip, and regular 256 (a group across a lane pair) on large
// problems.  Measured at 4096 x 3072 (B200, eight inputs back to back, L2
// not holding them): Sylvester 128 14.7 us against 16.8 us on the ring
// kernel; without rotation 15.8 against 10.6 and regular 256 18.6 against
// 16.8, so unrotated rows and small regular-256 problems stay on the ring
// kernel.  (The kernel template also implements the XOR-relabelled reads
// for the other rotations; the launcher does not instantiate them.)
// Regular 256 on the strip kernel from 2^25 elements up (measured on B200:
// 16384 x 3072 53.3 vs 55.3 us, 65536 x 12288 626.7 vs 792.6 us against the
// ring kernel; 4096 x 3072 22.5 vs 20.5 us, so small problems stay on the ring).
constexpr int64_t kStripReg256MinElems = (int64_t)1 << 25;
// QLIN_ROWQUANT_NO_HALF_STRIP=1 keeps Sylvester 128 on 128-element strips
// (comparison runs).
bool half_strip_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_ROWQUANT_NO_HALF_STRIP");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}
template <int DT>
int strip_by_rot(RotCode rc, const RowQuantParams& p, cudaStream_t s) {
  if (rc == RC_SYL128) {
    if (p.K / 64 <= 128 && !half_strip_disabled()) return launch_strip<DT, ROT_SYLVESTER, 128, 64>(p, s);
    return launch_strip<DT, ROT_SYLVESTER, 128>(p, s);
  }
  if (rc == RC_REG256 && (int64_t)p.M * p.K >= kStripReg256MinElems) return launch_strip<DT, ROT_REGULAR, 256>(p, s);
  return QLIN_ERR_UNSUPPORTED;
}

// QLIN_ROWQUANT_NO_STRIP=1 keeps 16-bit activations on the bulk-copy ring
// kernel (comparison runs).
bool strip_disabled() {
  static const bool off = [] {
    const char* v = getenv("QLIN_ROWQUANT_NO_STRIP");
    return v != nullptr && v[0] == '1';
  }();
  return off;
}

bool strip_ok(const RowQuantLaunch& L, const void* x, int64_t ldx, int64_t K, const int8_t* q) {
  return L.mode == MODE_INT8 && L.dt_in == L.dt_q && (L.dt_in == DT_BF16 || L.dt_in == DT_F16) && K % STRIP == 0 &&
         K / STRIP <= 128 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * 2) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(q) & 31) == 0 && !strip_disabled();
}

}  // namespace

int launch_rowquant(const RowQuantLaunch& L, const void* x, int64_t ldx, int64_t M, int64_t K, float rot_c,
                    float clamp_min, const float* in_scale, int in_scale_per_row, int8_t* q, float* scale,
                    void* out, uint64_t seed, cudaStream_t stream) {
  if (M == 0 || K == 0) return QLIN_OK;
  RowQuantParams p{};
  p.x = x;
  p.ldx = ldx;
  p.M = (int)M;
  p.K = (int)K;
  p.rot_c = rot_c;
  p.clamp_min = clamp_min;
  p.in_scale = in_scale;
  p.in_scale_per_row = in_scale_per_row;
  p.q = q;
  p.scale = scale;
  p.out = out;
  p.seed = seed;
  p.one = 1.0f;

  const RotCode rc = rot_code(L.rot_kind, L.rot_group);
  if (rc == RC_BAD) return fail(QLIN_ERR_UNSUPPORTED, "unsupported Hadamard kind/size");

  const int64_t nchunks = K / 16;
  if (nchunks > 2048) return fail(QLIN_ERR_UNSUPPORTED, "K > 32768 is not supported by the row kernels");
  // Activation int8 hot path: packed float32x2 kernel fed by a bulk-copy
  // ring (falls through to the register-prefetch kernel when two ring slots
  // do not fit in shared memory).
  if (strip_ok(L, x, ldx, K, q)) {
    const int rc2 = L.dt_in == DT_BF16 ? strip_by_rot<DT_BF16>(rc, p, stream) : strip_by_rot<DT_F16>(rc, p, stream);
    if (rc2 != QLIN_ERR_UNSUPPORTED) return rc2;
  }
  if (L.mode == MODE_INT8 && L.dt_in == L.dt_q) {
    int rc2 = QLIN_ERR_UNSUPPORTED;
    if (L.dt_in == DT_BF16) rc2 = x2_by_chunks<DT_BF16>(rc, p, (int)nchunks, stream);
    if (L.dt_in == DT_F16) rc2 = x2_by_chunks<DT_F16>(rc, p, (int)nchunks, stream);
    if (L.dt_in == DT_F32) rc2 = x2_by_chunks<DT_F32>(rc, p, (int)nchunks, stream);
    if (rc2 != QLIN_ERR_UNSUPPORTED) return rc2;
  }
  LaunchShape s;
  s.chunks = nchunks <= 1024 ? 1 : 2;
  const int64_t per = (nchunks + s.chunks - 1) / s.chunks;
  s.tpr = (int)(((per + 31) / 32) * 32);
  s.rpc = 256 / s.tpr;
  if (s.rpc < 1) s.rpc = 1;
  if (s.rpc > 32) s.rpc = 32;
  const bool staged = (rc == RC_REG64 || rc == RC_REG256 || rc == RC_SYL32 || rc == RC_SYL128);
  s.smem = staged ? (size_t)(s.rpc * s.tpr / 32) * 512 * sizeof(float) : 0;

  switch (L.dt_in) {
    case DT_BF16:
      if (L.dt_q == DT_BF16) return by_mode<DT_BF16, DT_BF16>(L.mode, rc, p, s, stream);
      if (L.dt_q == DT_F32) return by_mode<DT_BF16, DT_F32>(L.mode, rc, p, s, stream);
      break;
    case DT_F16:
      if (L.dt_q == DT_F16) return by_mode<DT_F16, DT_F16>(L.mode, rc, p, s, stream);
      if (L.dt_q == DT_F32) return by_mode<DT_F16, DT_F32>(L.mode, rc, p, s, stream);
      break;
    case DT_F32:
      if (L.dt_q == DT_F32) return by_mode<DT_F32, DT_F32>(L.mode, rc, p, s, stream);
      break;
    case DT_I8:
      if (L.dt_q == DT_F32) return by_mode<DT_I8, DT_F32>(L.mode, rc, p, s, stream);
      break;
    default: break;
  }
  return fail(QLIN_ERR_UNSUPPORTED, "unsupported input/compute dtype pair");
}

// Per-token int8 quantisation with the row norm / modulation prologue
// (16-bit inputs, K % 16 == 0, 16-byte aligned rows and vectors: checked by
// the caller).
int launch_rowquant_fused(int dt, int rot_kind, int rot_group, float rot_c, const void* x, int64_t ldx, int64_t M,
                          int64_t K, const FusedPrologue& f, int8_t* q, float* scale, cudaStream_t stream) {
  if (M == 0 || K == 0) return QLIN_OK;
  RowQuantParams p{};
  p.x = x;
  p.ldx = ldx;
  p.M = (int)M;
  p.K = (int)K;
  p.rot_c = rot_c;
  p.q = q;
  p.scale = scale;
  p.one = 1.0f;
  p.norm_kind = f.norm_kind;
  p.eps = f.eps;
  p.norm_w = f.norm_w;
  p.mod_mul = f.mod_mul;
  p.mul_ld = f.mul_ld;
  p.mod_add = f.mod_add;
  p.add_ld = f.add_ld;
  p.rows_per_sample = f.rows_per_sample > 0 ? f.rows_per_sample : M;
  const RotCode rc = rot_code(rot_kind, rot_kind == 0 ? 0 : rot_group);
  if (rc == RC_BAD) return fail(QLIN_ERR_UNSUPPORTED, "unsupported Hadamard kind/size");
  const int64_t nchunks = K / 16;
  if (nchunks > 2048) return fail(QLIN_ERR_UNSUPPORTED, "K > 32768 is not supported by the row kernels");
  int r = QLIN_ERR_UNSUPPORTED;
  if (dt == DT_BF16) r = x2_by_chunks<DT_BF16, true>(rc, p, (int)nchunks, stream);
  else if (dt == DT_F16) r = x2_by_chunks<DT_F16, true>(rc, p, (int)nchunks, stream);
  else return fail(QLIN_ERR_UNSUPPORTED, "the fused norm prologue takes bf16 or f16 input");
  if (r == QLIN_ERR_UNSUPPORTED) return fail(QLIN_ERR_UNSUPPORTED, "row too long for the fused norm prologue");
  return r;
}

// Per-token int8 quantisation of the SiTU activation of [hidden | gate] rows
// (16-bit inputs, K % 16 == 0, ldx >= 2K, 16-byte aligned rows: checked by
// the caller): the fused kernel with the SiTU prologue and no norm.
int launch_rowquant_situ(int dt, int rot_kind, int rot_group, float rot_c, const void* x, int64_t ldx, int64_t M,
                         int64_t K, int8_t* q, float* scale, cudaStream_t stream) {
  if (M == 0 || K == 0) return QLIN_OK;
  RowQuantParams p{};
  p.x = x;
  p.ldx = ldx;
  p.M = (int)M;
  p.K = (int)K;
  p.rot_c = rot_c;
  p.q = q;
  p.scale = scale;
  p.one = 1.0f;
  p.norm_kind = NORM_NONE;
  p.rows_per_sample = M;
  p.situ = 1;
  const RotCode rc = rot_code(rot_kind, rot_kind == 0 ? 0 : rot_group);
  if (rc == RC_BAD) return fail(QLIN_ERR_UNSUPPORTED, "unsupported Hadamard kind/size");
  const int64_t nchunks = K / 16;
  if (nchunks > 2048) return fail(QLIN_ERR_UNSUPPORTED, "K > 32768 is not supported by the row kernels");
  int r = QLIN_ERR_UNSUPPORTED;
  if (dt == DT_BF16) r = x2_by_chunks<DT_BF16, true>(rc, p, (int)nchunks, stream);
  else if (dt == DT_F16) r = x2_by_chunks<DT_F16, true>(rc, p, (int)nchunks, stream);
  else return fail(QLIN_ERR_UNSUPPORTED, "the SiTU prologue takes bf16 or f16 input");
  if (r == QLIN_ERR_UNSUPPORTED) return fail(QLIN_ERR_UNSUPPORTED, "row too long for the SiTU prologue");
  return r;
}

// Per-token int8 quantisation of concatenated rows [x1[r, 0:K1] | x2[r, 0:K2]]
// (16-bit or float32 inputs, K1 and K2 multiples of 16, 16-byte aligned
// sources and row strides: checked by the caller).  The two parts land next
// to each other in the ring slot, so the rotation groups may straddle them.
int launch_rowquant_cat(int dt, int rot_kind, int rot_group, float rot_c, const void* x1, int64_t ld1, int64_t K1,
                        const void* x2, int64_t ld2, int64_t K2, int64_t M, int8_t* q, float* scale,
                        cudaStream_t stream) {
  if (M == 0) return QLIN_OK;
  RowQuantParams p{};
  p.x = x1;
  p.ldx = ld1;
  p.x2 = x2;
  p.ldx2 = ld2;
  p.k1 = (int)K1;
  p.M = (int)M;
  p.K = (int)(K1 + K2);
  p.rot_c = rot_c;
  p.q = q;
  p.scale = scale;
  p.one = 1.0f;
  const RotCode rc = rot_code(rot_kind, rot_kind == 0 ? 0 : rot_group);
  if (rc == RC_BAD) return fail(QLIN_ERR_UNSUPPORTED, "unsupported Hadamard kind/size");
  const int64_t nchunks = p.K / 16;
  if (nchunks > 2048) return fail(QLIN_ERR_UNSUPPORTED, "K > 32768 is not supported by the row kernels");
  // 16-bit rows on the strip kernel (as launch_rowquant routes them), the
  // two parts landing side by side in its shared-memory row
  if ((dt == DT_BF16 || dt == DT_F16) && p.K % STRIP == 0 && p.K / STRIP <= 128 && K1 % 8 == 0 &&
      (reinterpret_cast<uintptr_t>(x1) & 15) == 0 && (reinterpret_cast<uintptr_t>(x2) & 15) == 0 &&
      (ld1 * 2) % 16 == 0 && (ld2 * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(q) & 31) == 0 && !strip_disabled()) {
    const int rs = dt == DT_BF16 ? strip_by_rot<DT_BF16>(rc, p, stream) : strip_by_rot<DT_F16>(rc, p, stream);
    if (rs != QLIN_ERR_UNSUPPORTED) return rs;
  }
  int r = QLIN_ERR_UNSUPPORTED;
  if (dt == DT_BF16) r = x2_by_chunks<DT_BF16>(rc, p, (int)nchunks, stream);
  else if (dt == DT_F16) r = x2_by_chunks<DT_F16>(rc, p, (int)nchunks, stream);
  else if (dt == DT_F32) r = x2_by_chunks<DT_F32>(rc, p, (int)nchunks, stream);
  if (r == QLIN_ERR_UNSUPPORTED) return fail(QLIN_ERR_UNSUPPORTED, "row too long for the concatenating quantiser");
  return r;
}

namespace {
// One thread waits, bounded, on an mbarrier phase that nothing completes.
__global__ void rq_wait_selftest_kernel() {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)rq_wait_bounded(&bar, 0);
}
}  // namespace

int launch_rowquant_wait_selftest(cudaStream_t stream) {
  rq_wait_selftest_kernel<<<1, 32, 0, stream>>>();
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QLIN_OK : cuda_fail(e, "row-kernel wait self-test launch");
}

int set_rowquant_wait_limit(uint64_t ns) {
  const cudaError_t e = cudaMemcpyToSymbol(g_rq_wait_limit_ns, &ns, sizeof(ns));
  return e == cudaSuccess ? QLIN_OK : cuda_fail(e, "set row-kernel wait limit");
}

// Error word of the row kernels: read and clear (bit 1: a bulk-copy wait
// timed out).
int read_rowquant_error(cudaStream_t stream, uint32_t* bits) {
  uint32_t h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_rq_error_bits, sizeof(uint32_t), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return cuda_fail(e, "read row-kernel error word");
  const uint32_t zero = 0;
  e = cudaMemcpyToSymbolAsync(g_rq_error_bits, &zero, sizeof(uint32_t), 0, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return cuda_fail(e, "clear row-kernel error word");
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "sync");
  *bits = h;
  return QLIN_OK;
}

// Unaligned rows (no rotation): generic kernel.
int launch_rowquant_generic(int dt, int mode, const void* x, int64_t ldx, int64_t M, int64_t K, float clamp_min,
                            int8_t* q, float* scale, cudaStream_t stream) {
  if (M == 0) return QLIN_OK;
  RowQuantParams p{};
  p.x = x;
  p.ldx = ldx;
  p.M = (int)M;
  p.K = (int)K;
  p.clamp_min = clamp_min;
  p.q = q;
  p.scale = scale;
  dim3 grid((unsigned)M), block(256);
#define QLIN_GEN(DTV, MV) rowquant_generic_kernel<DTV, MV><<<grid, block, 0, stream>>>(p)
  if (mode == MODE_INT8) {
    if (dt == DT_BF16) QLIN_GEN(DT_BF16, MODE_INT8);
    else if (dt == DT_F16) QLIN_GEN(DT_F16, MODE_INT8);
    else QLIN_GEN(DT_F32, MODE_INT8);
  } else {
    if (dt == DT_BF16) QLIN_GEN(DT_BF16, MODE_INT4_ROW);
    else if (dt == DT_F16) QLIN_GEN(DT_F16, MODE_INT4_ROW);
    else QLIN_GEN(DT_F32, MODE_INT4_ROW);
  }
#undef QLIN_GEN
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rowquant_generic launch");
  return QLIN_OK;
}

}  // namespace qlin
