// Attention prologue of a Flux-style DiT block, in place on the fused qkv
// projection rows: per-head RMSNorm of q and k followed by the rotary
// position embedding.  HBM bound: every q/k element is read once and
// written once (v is not touched); the norm weights and the cos/sin tables
// stay in L2.
#include <atomic>

#include "../../include/qlinear_b200.h"
#include "common.cuh"
#include "internal.h"

namespace qlin {
namespace {

struct QkParams {
  void* qkv;           // [rows, ld] in the dtype, row = [q heads | k heads | v heads]
  int64_t ld;          // row stride, elements
  int64_t rows;
  int heads;
  const void* q_w;     // RMSNorm weights [head_dim] in the dtype, or null
  const void* k_w;
  float eps;
  const float* cos_t;  // [positions, head_dim / 2] or null (no rotation)
  const float* sin_t;
  int64_t positions;   // token index of a row = row % positions
  float one;           // 1.0f at run time (see the rotary sum below)
};

template <int DT>
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == DT_BF16) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      const float2 f = __half22float2(h);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// A float pair rounded to the dtype and widened back (one packed conversion).
template <int DT>
__device__ __forceinline__ float2 round2(float2 v) {
  if constexpr (DT == DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    const uint32_t w = *reinterpret_cast<uint32_t*>(&h);
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    return __half22float2(__floats2half2_rn(v.x, v.y));
  }
}

template <int DT>
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == DT_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// LPV lanes per head vector (head_dim = 8 * LPV); each lane owns 8
// consecutive elements (one 16-byte load and store).  The q and k head
// vectors of all rows form one flat sequence (vector f is head vector
// f % (2 * heads) of row f / (2 * heads): q heads first, then k heads, so
// consecutive vectors are consecutive 16 * LPV-byte segments of a row).  A
// CTA covers V = U * (256 / LPV) consecutive vectors per iteration, one per
// slot (lane group g, k < U: vector g + k * 256 / LPV of the range), all U
// loads in flight before any is computed, and the grid strides by
// gridDim.x * V.  Each slot carries its (row, head vector, token position)
// from iteration to iteration by adding the stride's quotient and remainder
// (computed once), so the walk divides nothing per vector.
template <int DT, int LPV, int U>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(QkParams p) {
  pdl_wait();  // launched with PDL: the qkv rows of the previous kernel are visible
  pdl_launch_dependents();
  constexpr int HD = 8 * LPV;
  constexpr int G = 256 / LPV;  // lane groups per CTA
  constexpr int V = U * G;      // vectors per CTA and iteration
  const int sub = threadIdx.x % LPV;
  const int g = threadIdx.x / LPV;
  const int two_h = 2 * p.heads;
  const int64_t nvec = p.rows * two_h;
  const int64_t stride = (int64_t)gridDim.x * V;
  const int64_t st_rows = stride / two_h;           // the stride in rows ...
  const int st_hv = (int)(stride - st_rows * two_h);  // ... and head vectors
  const int64_t st_pos = st_rows % p.positions;
  int64_t row[U], pos[U];
  int hv[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t f = (int64_t)blockIdx.x * V + g + k * G;
    row[k] = f / two_h;
    hv[k] = (int)(f - row[k] * two_h);
    pos[k] = row[k] % p.positions;
  }
  // the loop bound is uniform across the CTA (shuffles need every lane)
  for (int64_t f0 = (int64_t)blockIdx.x * V; f0 < nvec; f0 += stride) {
    uint4 raw[U];
    int64_t off[U];
    bool ok[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      ok[k] = row[k] < p.rows;
      off[k] = row[k] * p.ld + (int64_t)hv[k] * HD + sub * 8;
      raw[k] = ok[k] ? __ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.qkv) + off[k]))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const bool is_k = hv[k] >= p.heads;
      float x[8];
      unpack8<DT>(raw[k], x);
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fmaf_rn(x[i], x[i], ss);
#pragma unroll
      for (int o = LPV / 2; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      // ss / HD is exact as a multiplication by the power of two 1 / HD
      const float rstd = __frsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / (float)HD), p.eps));
      const void* wp = is_k ? p.k_w : p.q_w;
      float w[8];
      if (wp != nullptr) {
        unpack8<DT>(*reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(wp) + sub * 8), w);
      }
      // element pairs (2j, 2j+1) in packed float32x2 arithmetic, each step
      // rounded as the scalar sequence: dt((x * rstd) * w), then the rotary
      // pair (c*a - s*b, s*a + c*b) with rounded products and sums
      const float2 r2 = make_float2(rstd, rstd);
      const float2 one2 = make_float2(p.one, p.one);
      float2 n2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 t = f2_mul(make_float2(x[2 * j], x[2 * j + 1]), r2);
        if (wp != nullptr) t = f2_mul(t, make_float2(w[2 * j], w[2 * j + 1]));
        n2[j] = round2<DT>(t);
      }
      if (p.cos_t != nullptr && ok[k]) {
        const float4 c4 = *reinterpret_cast<const float4*>(p.cos_t + pos[k] * (HD / 2) + sub * 4);
        const float4 s4 = *reinterpret_cast<const float4*>(p.sin_t + pos[k] * (HD / 2) + sub * 4);
        const float c[4] = {c4.x, c4.y, c4.z, c4.w};
        const float sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = n2[j].x, bb = n2[j].y;
          const float2 p0 = f2_mul(make_float2(c[j], sn[j]), make_float2(a, a));     // (c*a, s*a)
          const float2 p1 = f2_mul(make_float2(-sn[j], c[j]), make_float2(bb, bb));  // (-s*b, c*b)
          // the sum as an FMA by a run-time 1.0: the assembler fuses a packed
          // multiply with a following packed add into one FMA (one rounding)
          // even with .rn on both, which would change the result
          n2[j] = f2_fma(p1, one2, p0);
        }
      }
      float n[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        n[2 * j] = n2[j].x;
        n[2 * j + 1] = n2[j].y;
      }
      if (ok[k]) __stcs(reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.qkv) + off[k]), pack8<DT>(n));
    }
    // next vector of each slot: stride = st_rows rows + st_hv head vectors
#pragma unroll
    for (int k = 0; k < U; ++k) {
      hv[k] += st_hv;
      int64_t dr = st_rows, dp = st_pos;
      if (hv[k] >= two_h) {
        hv[k] -= two_h;
        dr += 1;
        dp += 1;
      }
      row[k] += dr;
      pos[k] += dp;
      while (pos[k] >= p.positions) pos[k] -= p.positions;  // dp <= positions: at most twice
    }
  }
}

template <int DT, int LPV>
int launch_qk(const QkParams& p, cudaStream_t stream) {
  constexpr int U = 4;
  const int64_t vecs = p.rows * 2 * p.heads;
  const int64_t per_block = (256 / LPV) * U;
  int64_t blocks = (vecs + per_block - 1) / per_block;
  auto kern = qk_norm_rope_kernel<DT, LPV, U>;
  static std::atomic<int> per_sm{0};  // resident CTAs per SM (one device model per process)
  if (per_sm.load() == 0) {
    int nb = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, 256, 0);
    if (e != cudaSuccess) return cuda_fail(e, "occupancy query");
    per_sm.store(nb > 0 ? nb : 1);
  }
  const int64_t cap = (int64_t)device_sm_count() * per_sm.load();  // one wave of resident CTAs
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cudaError_t e = launch_pdl(kern, dim3((unsigned)blocks), dim3(256), 0, stream, p);
  if (e != cudaSuccess) return cuda_fail(e, "qk_norm_rope launch");
  return QLIN_OK;
}

}  // namespace

int launch_qk_norm_rope(int dt, void* qkv, int64_t rows, int64_t ld, int heads, int head_dim, const void* q_w,
                        const void* k_w, float eps, const float* cos_t, const float* sin_t, int64_t positions,
                        cudaStream_t stream) {
  if (rows == 0 || heads == 0) return QLIN_OK;
  QkParams p{qkv, ld, rows, heads, q_w, k_w, eps, cos_t, sin_t, positions > 0 ? positions : rows, 1.0f};
  if (dt == DT_BF16) {
    if (head_dim == 128) return launch_qk<DT_BF16, 16>(p, stream);
    if (head_dim == 64) return launch_qk<DT_BF16, 8>(p, stream);
  } else if (dt == DT_F16) {
    if (head_dim == 128) return launch_qk<DT_F16, 16>(p, stream);
    if (head_dim == 64) return launch_qk<DT_F16, 8>(p, stream);
  }
  return fail(QLIN_ERR_UNSUPPORTED, "qk_norm_rope supports bf16/f16 and head_dim 64 or 128");
}

}  // namespace qlin
