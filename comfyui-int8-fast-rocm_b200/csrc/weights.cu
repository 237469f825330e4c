// Weight-format kernels that are not row rotations: asymmetric W4A8
// (Lloyd-Max codebook) dequantisation fused with per-channel int8
// requantisation.
#include <cuda_fp8.h>

#include "../../include/qlinear_b200.h"
#include "common.cuh"
#include "internal.h"

namespace qlin {
namespace {

// One row per CTA; each thread owns 16 consecutive k (8 packed bytes).
// w[n,k] = (codebook[code] * s_channel[n]) * s_rel[n, k / gs]  (w4a8_int8.py:46-75)
// then either (wout != null) the float32 row itself, or
// quantize_int8_axiswise(dim=1): absmax/127 clamped at 1e-30, rint(w * (1/s)).
__global__ void __launch_bounds__(1024) requant_asym_w4a8_kernel(const uint8_t* __restrict__ packed,
                                                                   const float* __restrict__ codebook,
                                                                   const float* __restrict__ s_channel,
                                                                   const uint8_t* __restrict__ s_rel, int gs,
                                                                   int N, int K, int8_t* __restrict__ q,
                                                                   float* __restrict__ scale,
                                                                   float* __restrict__ wout) {
  __shared__ float cb[16];
  __shared__ float red[32];
  const int n = blockIdx.x;
  const int t = threadIdx.x;
  if (t < 16) cb[t] = codebook[t];
  __syncthreads();
  const int nchunks = K >> 4;
  const bool active = t < nchunks;
  float v[16];
  const float sch = s_channel[n];
  const int ngroups = K / gs;
  if (active) {
    const uint2 pk = *reinterpret_cast<const uint2*>(packed + (int64_t)n * (K >> 1) + t * 8);
    const uint32_t w2[2] = {pk.x, pk.y};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int code = (w2[j >> 3] >> (4 * (j & 7))) & 0xF;  // low nibble = even k
      const int k = t * 16 + j;
      __nv_fp8_e4m3 f8;
      f8.__x = s_rel[(int64_t)n * ngroups + k / gs];
      const float sr = static_cast<float>(f8);
      v[j] = __fmul_rn(__fmul_rn(cb[code], sch), sr);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = 0.0f;
  }
  if (wout != nullptr) {  // float32 dequantisation only (uniform over the grid)
    if (active) {
      float4* d = reinterpret_cast<float4*>(wout + (int64_t)n * K + t * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    return;
  }
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) a = fmaxf(a, fabsf(v[j]));
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((t & 31) == 0) red[t >> 5] = a;
  __syncthreads();
  a = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a = fmaxf(a, red[w]);
  const float s = fmaxf(__fdiv_rn(a, 127.0f), 1e-30f);
  const float inv = __frcp_rn(s);
  if (t == 0) scale[n] = s;
  if (!active) return;
  uint32_t o[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float y = fminf(fmaxf(__fmul_rn(v[4 * w + b], inv), -128.0f), 127.0f);
      word |= ((uint32_t)rint_to_int(y) & 0xFFu) << (8 * b);
    }
    o[w] = word;
  }
  *reinterpret_cast<uint4*>(q + (int64_t)n * K + t * 16) = make_uint4(o[0], o[1], o[2], o[3]);
}

// SiTU gated activation on [hidden | gate] rows (int8_fused_kernel.py:403-421):
// out = situ_f(h, g), one element per thread.
template <int DT>
__global__ void __launch_bounds__(256) situ_kernel(const void* __restrict__ x, int64_t ldx, int M, int K,
                                                   void* __restrict__ y) {
  using E = Elem<DT>;
  using T = typename E::T;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * K) return;
  const int64_t row = idx / K;
  const int col = (int)(idx - row * K);
  const T* xr = reinterpret_cast<const T*>(x) + row * ldx;
  const float h = E::to_f(xr[col]);
  const float g = E::to_f(xr[K + col]);
  reinterpret_cast<T*>(y)[row * K + col] = E::from_f(situ_f(h, g));
}

}  // namespace

int launch_situ(int dt, const void* x, int64_t ldx, int64_t M, int64_t K, void* y, cudaStream_t stream) {
  const int64_t n = M * K;
  if (n == 0) return QLIN_OK;
  const unsigned grid = (unsigned)((n + 255) / 256);
  if (dt == DT_BF16) situ_kernel<DT_BF16><<<grid, 256, 0, stream>>>(x, ldx, (int)M, (int)K, y);
  else if (dt == DT_F16) situ_kernel<DT_F16><<<grid, 256, 0, stream>>>(x, ldx, (int)M, (int)K, y);
  else situ_kernel<DT_F32><<<grid, 256, 0, stream>>>(x, ldx, (int)M, (int)K, y);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "situ launch");
  return QLIN_OK;
}

int launch_requant_asym_w4a8(const uint8_t* packed, const float* codebook, const float* s_channel,
                             const uint8_t* s_rel, int group_size, int64_t N, int64_t K, int8_t* q, float* scale,
                             float* wout, cudaStream_t stream) {
  if (K > 16384) return fail(QLIN_ERR_UNSUPPORTED, "asym W4A8 kernels support K <= 16384");
  const int threads = (int)(((K / 16) + 31) / 32 * 32);
  requant_asym_w4a8_kernel<<<(unsigned)N, threads, 0, stream>>>(packed, codebook, s_channel, s_rel, group_size,
                                                                 (int)N, (int)K, q, scale, wout);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "requant_asym_w4a8 launch");
  return QLIN_OK;
}

}  // namespace qlin
