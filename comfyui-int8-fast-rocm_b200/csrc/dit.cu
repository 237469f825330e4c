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
  constexpr int HD = 8 * LPV;
  const int sub = threadIdx.x % LPV;
  const int64_t groups_total = (int64_t)gridDim.x * (blockDim.x / LPV);
  const int64_t g0 = (int64_t)blockIdx.x * (blockDim.x / LPV) + threadIdx.x / LPV;
  const int two_h = 2 * p.heads;
  const int64_t nvec = p.rows * two_h;
  // the loop bound is uniform across the warp (shuffles need every lane)
  const int64_t warp_first = g0 - (threadIdx.x % 32) / LPV;
  for (int64_t base = warp_first; base < nvec; base += groups_total * U) {
    const int64_t my0 = base + (g0 - warp_first);
    uint4 raw[U];
    int64_t off[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = my0 + (int64_t)u * groups_total;
      ok[u] = v < nvec;
      const int64_t row = ok[u] ? v / two_h : 0;
      const int hv = ok[u] ? (int)(v - row * two_h) : 0;
      off[u] = row * p.ld + (int64_t)hv * HD + sub * 8;
      raw[u] = ok[u] ? __ldcs(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.qkv) + off[u]))
                     : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = my0 + (int64_t)u * groups_total;
      const int64_t row = ok[u] ? v / two_h : 0;
      const bool is_k = ok[u] && (int)(v - row * two_h) >= p.heads;
      float x[8];
      unpack8<DT>(raw[u], x);
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fmaf_rn(x[i], x[i], ss);
#pragma unroll
      for (int o = LPV / 2; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      const float rstd = __frsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), p.eps));
      const void* wp = is_k ? p.k_w : p.q_w;
      float w[8];
      if (wp != nullptr) {
        unpack8<DT>(*reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(wp) + sub * 8), w);
      }
      float n[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float t = __fmul_rn(x[i], rstd);
        n[i] = Elem<DT>::round(wp != nullptr ? __fmul_rn(t, w[i]) : t);
      }
      if (p.cos_t != nullptr) {
        const int64_t pos = row % p.positions;
        const float4 c4 = *reinterpret_cast<const float4*>(p.cos_t + pos * (HD / 2) + sub * 4);
        const float4 s4 = *reinterpret_cast<const float4*>(p.sin_t + pos * (HD / 2) + sub * 4);
        const float c[4] = {c4.x, c4.y, c4.z, c4.w};
        const float s[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float a = n[2 * j], b = n[2 * j + 1];
          n[2 * j] = __fsub_rn(__fmul_rn(c[j], a), __fmul_rn(s[j], b));
          n[2 * j + 1] = __fadd_rn(__fmul_rn(s[j], a), __fmul_rn(c[j], b));
        }
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
  qk_norm_rope_kernel<DT, LPV, U><<<(unsigned)blocks, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "qk_norm_rope launch");
  return QLIN_OK;
}

}  // namespace

int launch_qk_norm_rope(int dt, void* qkv, int64_t rows, int64_t ld, int heads, int head_dim, const void* q_w,
                        const void* k_w, float eps, const float* cos_t, const float* sin_t, int64_t positions,
                        cudaStream_t stream) {
  if (rows == 0 || heads == 0) return QLIN_OK;
  QkParams p{qkv, ld, rows, heads, q_w, k_w, eps, cos_t, sin_t, positions > 0 ? positions : rows};
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
