// Attention prologue of a Flux-style DiT block, in place on the fused qkv
// projection rows: per-head RMSNorm of q and k followed by the rotary
// position embedding.  HBM bound: every q/k element is read once and
// written once (v is not touched); the norm weights and the cos/sin tables
// stay in L2.
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
// consecutive elements (one 16-byte load and store).  Vector v of the
// grid-stride walk is head vector v % (2 * heads) of row v / (2 * heads):
// q heads first, then k heads, i.e. the column offset is (v % 2H) * head_dim,
// so the lanes of a warp cover 512 contiguous bytes.  U vectors per lane
// group are loaded before any is computed.
template <int DT, int LPV, int U>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(QkParams p) {
  pdl_wait();  // launched with PDL: the qkv rows of the previous kernel are visible
  pdl_launch_dependents();
  constexpr int HD = 8 * LPV;
  const int sub = threadIdx.x % LPV;
  const int64_t groups_total = (int64_t)gridDim.x * (blockDim.x / LPV);
  const int64_t g0 = (int64_t)blockIdx.x * (blockDim.x / LPV) + threadIdx.x / LPV;
  const int two_h = 2 * p.heads;
  const int64_t nvec = p.rows * two_h;
  const bool small = nvec + groups_total * U < ((int64_t)1 << 32);
  // the loop bound is uniform across the warp (shuffles need every lane)
  const int64_t warp_first = g0 - (threadIdx.x % 32) / LPV;
  for (int64_t base = warp_first; base < nvec; base += groups_total * U) {
    const int64_t my0 = base + (g0 - warp_first);
    uint4 raw[U];
    int64_t off[U], rows_u[U];
    int hvs[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = my0 + (int64_t)u * groups_total;
      ok[u] = v < nvec;
      // 32-bit division when the vector index fits (a 64-bit one is a long
      // emulated sequence)
      const int64_t row = !ok[u] ? 0 : (small ? (int64_t)((uint32_t)v / (uint32_t)two_h) : v / two_h);
      const int hv = ok[u] ? (int)(v - row * two_h) : 0;
      rows_u[u] = row;
      hvs[u] = hv;
      off[u] = row * p.ld + (int64_t)hv * HD + sub * 8;
      raw[u] = ok[u] ? __ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.qkv) + off[u]))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = rows_u[u];
      const bool is_k = ok[u] && hvs[u] >= p.heads;
      float x[8];
      unpack8<DT>(raw[u], x);
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
      if (p.cos_t != nullptr) {
        const int64_t pos = row % p.positions;
        const float4 c4 = *reinterpret_cast<const float4*>(p.cos_t + pos * (HD / 2) + sub * 4);
        const float4 s4 = *reinterpret_cast<const float4*>(p.sin_t + pos * (HD / 2) + sub * 4);
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
      if (ok[u]) __stcs(reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.qkv) + off[u]), pack8<DT>(n));
    }
  }
}

template <int DT, int LPV>
int launch_qk(const QkParams& p, cudaStream_t stream) {
  constexpr int U = 2;
  const int64_t groups = p.rows * 2 * p.heads;
  const int64_t per_block = 256 / LPV;
  int64_t blocks = (groups + per_block * U - 1) / (per_block * U);
  const int64_t cap = (int64_t)device_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cudaError_t e = launch_pdl(qk_norm_rope_kernel<DT, LPV, U>, dim3((unsigned)blocks), dim3(256), 0, stream, p);
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
