// Row-wise rotate + quantise kernels (bandwidth bound).
//
// One warp covers 32 consecutive 16-element chunks of a row; a row is covered
// by TPR threads (a multiple of 32), a CTA holds RPC rows.  Every thread
// keeps its CHUNKS x 16 elements in registers from the single HBM read to
// the single HBM write:
//   1. 128-bit loads, convert to float32 (int8 input: times its row scale);
//   2. ConvRot stage 1: Hadamard digits inside the 16-element chunk;
//   3. ConvRot stage 2 (group > 16): the chunk-index digits, through a
//      per-warp swizzled shared-memory transpose (only __syncwarp needed:
//      a rotation group never leaves its warp);
//   4. times the normalisation constant, rounded to the compute dtype;
//   5. absmax (row: warp shuffles + one CTA exchange; group of 128: 8 lanes),
//      scale and codes with the reference's exact rounding sequence;
//   6. one 128-bit (or 64-bit packed-int4) store per chunk.
#pragma once

#include "common.cuh"

namespace qlin {

enum : int {
  MODE_INT8 = 0,        // quantize_int8_axiswise(dim=-1): absmax/127, rint(x * (1/s))
  MODE_INT4_ROW = 1,    // quantize_signed_int4_rowwise: dtype math, codes in [-7, 7]
  MODE_INT4_G128 = 2,   // same conventions per 128-element group
  MODE_ROTATE = 3,      // rotated values only, in the compute dtype
  MODE_REQUANT = 4,     // quantize_int8(x, given scale), round-half-even
  MODE_REQUANT_SR = 5,  // stochastic rounding with a given scale
};
enum : int { DT_I8 = 3 };  // extra input type for dequantisation

struct RowQuantParams {
  const void* x;
  int64_t ldx;           // input row stride, elements
  int M, K;
  float rot_c;           // normalised Hadamard entry in the compute dtype
  float clamp_min;       // int4: 1e-10 in the compute dtype
  const float* in_scale; // int8 input (dequant) or given requant scale
  int in_scale_per_row;  // 1: in_scale[M], 0: in_scale[0]
  int8_t* q;             // codes: [M, K] int8
  float* scale;          // per-row [M] or per-group [M, K/128]
  void* out;             // MODE_ROTATE output [M, K] in the compute dtype,
                         // or packed int4 codes [M, K/2] for the int4 modes
  uint64_t seed;         // MODE_REQUANT_SR
  float one;             // 1.0f, unknown to the compiler (see rowquant_pair_kernel)
  // fused prologue of rowquant_x2_kernel<..., FUSED = true> (input dtype):
  //   y = dt(norm(x)); y = dt(y * mod_mul[s, k]); y = dt(y + mod_add[s, k])
  // with s = row / rows_per_sample; then rotation and quantisation of y
  int norm_kind;         // NORM_NONE / NORM_LAYER / NORM_RMS
  float eps;
  const void* norm_w;    // NORM_RMS weight [K] or null
  const void* mod_mul;   // [S, mul_ld] or null
  int64_t mul_ld;
  const void* mod_add;   // [S, add_ld] or null
  int64_t add_ld;
  int64_t rows_per_sample;
  // second source of rowquant_x2_kernel (x2 != null): row r is the
  // concatenation [x[r, 0:k1] | x2[r, 0:K-k1]], x2 rows ldx2 elements apart
  const void* x2;
  int64_t ldx2;
  int k1;
  // SiTU prologue of rowquant_x2_kernel<..., FUSED = true>: source row r is
  // [hidden[r, 0:K] | gate[r, 0:K]] (x, ldx >= 2K elements); the row
  // quantised is dt(situ_f(hidden, gate))
  int situ;
};

enum : int {
  NORM_NONE = 0,
  NORM_LAYER = 1,  // (x - mean) * rsqrt(var + eps), no affine (F.layer_norm without weight)
  NORM_RMS = 2,    // (x * rsqrt(mean(x^2) + eps)) * weight, rounded once (F.rms_norm)
};

// Swizzled float index inside a warp's 512-float staging buffer.  XORs the
// low three bits of the 16-byte chunk index with bits of the chunk index
// above them, so both the natural-order float4 accesses and the transposed
// stage-2 accesses of each rotation size are (nearly) bank-conflict free.
template <int R>
__device__ __forceinline__ int swz(int e) {
  constexpr int S = (R >= 16) ? 6 : (R == 8) ? 5 : (R == 4) ? 4 : 3;
  const int c = e >> 2;
  const int p = c ^ ((c >> 3) & 3) ^ (((c >> S) & 1) << 2);
  return (p << 2) | (e & 3);
}

// Counter-based uniform random in [0, 1) (SplitMix64 finaliser of
// seed + element index); 24 random bits.
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t idx) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull * (idx + 1);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(uint32_t)(z >> 40) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  const uint32_t ab = __byte_perm((uint32_t)a, (uint32_t)b, 0x0040);
  const uint32_t cd = __byte_perm((uint32_t)c, (uint32_t)d, 0x0040);
  return __byte_perm(ab, cd, 0x5410);
}

// Raw 16-element chunk as loaded from HBM (converted to float only when
// used, so a prefetched row costs 8 registers for 16-bit inputs).
template <int DT_IN>
struct RawChunk {
  static constexpr int WORDS = DT_IN == DT_F32 ? 16 : (DT_IN == DT_I8 ? 4 : 8);
  uint32_t w[WORDS];
};

template <int DT_IN>
__device__ __forceinline__ void load_raw(const void* base, int64_t off, RawChunk<DT_IN>& r) {
  constexpr int BYTES = DT_IN == DT_F32 ? 4 : (DT_IN == DT_I8 ? 1 : 2);
  const uint4* q = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(base) + off * BYTES);
#pragma unroll
  for (int i = 0; i < RawChunk<DT_IN>::WORDS / 4; ++i) {
    const uint4 t = __ldg(q + i);
    r.w[4 * i] = t.x; r.w[4 * i + 1] = t.y; r.w[4 * i + 2] = t.z; r.w[4 * i + 3] = t.w;
  }
}

template <int DT_IN>
__device__ __forceinline__ void unpack_raw(const RawChunk<DT_IN>& r, float (&v)[16], float s) {
  if constexpr (DT_IN == DT_F32) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r.w[j]);
  } else if constexpr (DT_IN == DT_BF16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[2 * j] = __uint_as_float(r.w[j] << 16);
      v[2 * j + 1] = __uint_as_float(r.w[j] & 0xFFFF0000u);
    }
  } else if constexpr (DT_IN == DT_F16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.w[j]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int b = (int)(int8_t)((r.w[j >> 2] >> (8 * (j & 3))) & 0xFF);
      v[j] = __fmul_rn((float)b, s);  // dequantize: q.float() * scale
    }
  }
}

// Round 16 floats to the compute dtype in pairs (one packed conversion per
// pair), returning the rounded values as float.
template <int DT>
__device__ __forceinline__ void round16(float (&v)[16]) {
  if constexpr (DT == DT_BF16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
      const uint32_t u = *reinterpret_cast<uint32_t*>(&h);
      v[2 * j] = __uint_as_float(u << 16);
      v[2 * j + 1] = __uint_as_float(u & 0xFFFF0000u);
    }
  } else if constexpr (DT == DT_F16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 f = __half22float2(__floats2half2_rn(v[2 * j], v[2 * j + 1]));
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
    }
  }
}

// max(a, b) that returns NaN when either operand is NaN (torch's amax
// propagates NaN; fmaxf would drop it).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Persistent row loop: each CTA walks rows blockIdx.x*RPC + k*gridDim.x*RPC,
// prefetching the next row's chunks into registers while the current one is
// rotated and quantised; per-thread shared-memory offsets are computed once.
template <int DT_IN, int DT_Q, int KIND, int R, int CHUNKS, int MODE>
__global__ void __launch_bounds__(1024) rowquant_kernel(RowQuantParams p) {
  using EQ = Elem<DT_Q>;
  extern __shared__ float stage_smem[];  // [warps][512] when R > 1
  __shared__ float red[2][32][33];       // [iteration parity][row][warp] partial absmax

  const int tpr = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31;
  const int warp_in_row = t >> 5;
  const int nchunks = p.K >> 4;
  const int warp_lin = threadIdx.y * (tpr >> 5) + warp_in_row;
  float* wbuf = stage_smem + warp_lin * 512;
  (void)wbuf;

  // ConvRot stage-2 offsets (floats): natural order (4 float4 of this lane's
  // chunk) and the transposed column set (R rows x J floats, J2-wide vectors).
  constexpr int J = 16 / R;
  constexpr int J2 = J < 4 ? J : 4;
  constexpr int NQ = J / J2;
  int nat[4];
  int s2[R > 1 ? R : 1][NQ];
  if constexpr (KIND != ROT_NONE && R > 1) {
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) nat[q4] = swz<R>(lane * 16 + 4 * q4);
    const int g0 = (lane / R) * (16 * R);
    const int rp = lane % R;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int q = 0; q < NQ; ++q) s2[r][q] = swz<R>(g0 + 16 * r + rp * J + q * J2);
  }

  const int rows_per_cta = blockDim.y;
  const int stride_rows = gridDim.x * rows_per_cta;
  RawChunk<DT_IN> raw[CHUNKS];
  int first = blockIdx.x * rows_per_cta;
  {
    const int row = first + threadIdx.y;
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const int ci = t + i * tpr;
      if (row < p.M && ci < nchunks) load_raw<DT_IN>(p.x, (int64_t)row * p.ldx + (int64_t)ci * 16, raw[i]);
    }
  }

  for (int it = 0; first < p.M; ++it, first += stride_rows) {
    const int row = first + threadIdx.y;
    const bool row_ok = row < p.M;
    float in_s = 1.0f;
    if constexpr (DT_IN == DT_I8) {
      if (row_ok) in_s = p.in_scale_per_row ? __ldg(p.in_scale + row) : __ldg(p.in_scale);
    }
    float v[CHUNKS][16];
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const int ci = t + i * tpr;
      if (row_ok && ci < nchunks) {
        unpack_raw<DT_IN>(raw[i], v[i], in_s);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[i][j] = 0.0f;
      }
    }
    // prefetch the next row handled by this thread
    {
      const int nrow = row + stride_rows;
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        const int ci = t + i * tpr;
        if (nrow < p.M && ci < nchunks) load_raw<DT_IN>(p.x, (int64_t)nrow * p.ldx + (int64_t)ci * 16, raw[i]);
      }
    }

    if constexpr (KIND != ROT_NONE) {
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        xform_regs<KIND, 16>(v[i]);
        if constexpr (R > 1) {
          // stage 2: Hadamard over the chunk index within each group of R chunks
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            *reinterpret_cast<float4*>(wbuf + nat[q4]) =
                make_float4(v[i][4 * q4], v[i][4 * q4 + 1], v[i][4 * q4 + 2], v[i][4 * q4 + 3]);
          __syncwarp();
          float w[J][R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
              if constexpr (J2 == 4) {
                const float4 f = *reinterpret_cast<const float4*>(wbuf + s2[r][q]);
                w[4 * q][r] = f.x; w[4 * q + 1][r] = f.y; w[4 * q + 2][r] = f.z; w[4 * q + 3][r] = f.w;
              } else if constexpr (J2 == 2) {
                const float2 f = *reinterpret_cast<const float2*>(wbuf + s2[r][q]);
                w[0][r] = f.x; w[1][r] = f.y;
              } else {
                w[0][r] = wbuf[s2[r][q]];
              }
            }
          }
#pragma unroll
          for (int jj = 0; jj < J; ++jj) xform_regs<KIND, R>(w[jj]);
#pragma unroll
          for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
              if constexpr (J2 == 4) {
                *reinterpret_cast<float4*>(wbuf + s2[r][q]) =
                    make_float4(w[4 * q][r], w[4 * q + 1][r], w[4 * q + 2][r], w[4 * q + 3][r]);
              } else if constexpr (J2 == 2) {
                *reinterpret_cast<float2*>(wbuf + s2[r][q]) = make_float2(w[0][r], w[1][r]);
              } else {
                wbuf[s2[r][q]] = w[0][r];
              }
            }
          }
          __syncwarp();
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 f = *reinterpret_cast<const float4*>(wbuf + nat[q4]);
            v[i][4 * q4] = f.x; v[i][4 * q4 + 1] = f.y; v[i][4 * q4 + 2] = f.z; v[i][4 * q4 + 3] = f.w;
          }
          __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) v[i][j] = __fmul_rn(v[i][j], p.rot_c);
        round16<DT_Q>(v[i]);
      }
    }

    if constexpr (MODE == MODE_ROTATE) {
      if (row_ok) {
        auto* out = reinterpret_cast<typename EQ::T*>(p.out) + (int64_t)row * p.K;
#pragma unroll
        for (int i = 0; i < CHUNKS; ++i) {
          const int ci = t + i * tpr;
          if (ci < nchunks) store16<DT_Q>(out + (int64_t)ci * 16, v[i]);
        }
      }
      continue;
    } else if constexpr (MODE == MODE_REQUANT || MODE == MODE_REQUANT_SR) {
      if (!row_ok) continue;
      const float s = p.in_scale_per_row ? __ldg(p.in_scale + row) : __ldg(p.in_scale);
      const float inv = __frcp_rn(s);
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        const int ci = t + i * tpr;
        if (ci >= nchunks) continue;
        int qv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          float y;
          if constexpr (MODE == MODE_REQUANT) {
            y = __fmul_rn(v[i][j], inv);                       // x * (1/scale)
            y = (y != y) ? 0.0f : fminf(fmaxf(y, -128.0f), 127.0f);
            qv[j] = rint_to_int(y);
          } else {
            const float xs = __fdiv_rn(v[i][j], s);            // x / scale
            const float fl = floorf(xs);
            const float frac = __fsub_rn(xs, fl);
            const float u = uniform01(p.seed, (uint64_t)row * p.K + ci * 16 + j);
            y = (u < frac) ? __fadd_rn(fl, 1.0f) : fl;
            y = (y != y) ? 0.0f : fminf(fmaxf(y, -128.0f), 127.0f);
            qv[j] = (int)y;
          }
        }
        int4 o;
        o.x = (int)pack4(qv[0], qv[1], qv[2], qv[3]);
        o.y = (int)pack4(qv[4], qv[5], qv[6], qv[7]);
        o.z = (int)pack4(qv[8], qv[9], qv[10], qv[11]);
        o.w = (int)pack4(qv[12], qv[13], qv[14], qv[15]);
        *reinterpret_cast<int4*>(p.q + (int64_t)row * p.K + (int64_t)ci * 16) = o;
      }
      continue;
    } else {
      // ---- absmax ----
      float amax_row = 0.0f;
      float amax_grp[CHUNKS];
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        float a = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) a = fmax_nan(a, fabsf(v[i][j]));
        amax_grp[i] = a;
        amax_row = fmax_nan(amax_row, a);
      }
      if constexpr (MODE == MODE_INT4_G128) {
#pragma unroll
        for (int i = 0; i < CHUNKS; ++i) {
#pragma unroll
          for (int o = 1; o < 8; o <<= 1) amax_grp[i] = fmax_nan(amax_grp[i], __shfl_xor_sync(0xffffffffu, amax_grp[i], o));
        }
      } else {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax_row = fmax_nan(amax_row, __shfl_xor_sync(0xffffffffu, amax_row, o));
        const int nw = tpr >> 5;
        float (*rb)[33] = red[it & 1];
        if (lane == 0) rb[threadIdx.y][warp_in_row] = amax_row;
        __syncthreads();
        amax_row = rb[threadIdx.y][0];
        for (int w2 = 1; w2 < nw; ++w2) amax_row = fmax_nan(amax_row, rb[threadIdx.y][w2]);
      }
      if (!row_ok) continue;

      float s_row = 0.0f, inv_row = 0.0f;
      if constexpr (MODE == MODE_INT8) {
        if (!(amax_row < __uint_as_float(0x7F800000u))) {
          // Inf or NaN in the row: the reference's scale is Inf / NaN, every
          // code is a NaN or 0 product and casts to 0.
          if (t == 0) p.scale[row] = amax_row;
#pragma unroll
          for (int i = 0; i < CHUNKS; ++i) {
            const int ci = t + i * tpr;
            if (ci < nchunks)
              *reinterpret_cast<int4*>(p.q + (int64_t)row * p.K + (int64_t)ci * 16) = make_int4(0, 0, 0, 0);
          }
          continue;
        }
        s_row = fmaxf(__fdiv_rn(amax_row, 127.0f), 1e-30f);  // (absmax.float()/127).clamp(1e-30)
        inv_row = __frcp_rn(s_row);                           // 1.0 / scale
        if (t == 0) p.scale[row] = s_row;
      } else if constexpr (MODE == MODE_INT4_ROW) {
        s_row = EQ::round(__fdiv_rn(fmaxf(amax_row, p.clamp_min), 7.0f));
        if (t == 0) p.scale[row] = s_row;
      }

#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        const int ci = t + i * tpr;
        if (ci >= nchunks) continue;
        if constexpr (MODE == MODE_INT8) {
          // |v| <= absmax, so |v * (1/scale)| <= 127 * (1 + 3 ulp) and the
          // round-half-even code is already in [-127, 127]: no clamp needed.
          // The low byte of (y + 1.5*2^23) is the two's-complement code.
          uint32_t u[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) u[j] = __float_as_uint(__fadd_rn(__fmul_rn(v[i][j], inv_row), 12582912.0f));
          int4 o;
          o.x = (int)pack4((int)u[0], (int)u[1], (int)u[2], (int)u[3]);
          o.y = (int)pack4((int)u[4], (int)u[5], (int)u[6], (int)u[7]);
          o.z = (int)pack4((int)u[8], (int)u[9], (int)u[10], (int)u[11]);
          o.w = (int)pack4((int)u[12], (int)u[13], (int)u[14], (int)u[15]);
          *reinterpret_cast<int4*>(p.q + (int64_t)row * p.K + (int64_t)ci * 16) = o;
        } else {
          float s = s_row;
          if constexpr (MODE == MODE_INT4_G128) {
            s = EQ::round(__fdiv_rn(fmaxf(amax_grp[i], p.clamp_min), 7.0f));
            if ((ci & 7) == 0) p.scale[(int64_t)row * (p.K >> 7) + (ci >> 3)] = s;
          }
          int qv[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float y = EQ::round(__fdiv_rn(v[i][j], s));  // (x / scale) in the compute dtype
            // NaN (0/0 on an all-zero row in f16, where the 1e-10 clamp
            // underflows) converts to code 0, as torch's float->int8 cast does
            y = (y != y) ? 0.0f : fminf(fmaxf(y, -7.0f), 7.0f);
            qv[j] = rint_to_int(y);
          }
          if (p.out != nullptr) {
            // packed int4 output [M, K/2]: low nibble = even k
            uint32_t w2[2] = {0u, 0u};
#pragma unroll
            for (int j = 0; j < 16; ++j) w2[j >> 3] |= ((uint32_t)qv[j] & 0xFu) << (4 * (j & 7));
            *reinterpret_cast<uint2*>(reinterpret_cast<int8_t*>(p.out) + (int64_t)row * (p.K >> 1) +
                                      (int64_t)ci * 8) = make_uint2(w2[0], w2[1]);
          } else {
            int4 o;
            o.x = (int)pack4(qv[0], qv[1], qv[2], qv[3]);
            o.y = (int)pack4(qv[4], qv[5], qv[6], qv[7]);
            o.z = (int)pack4(qv[8], qv[9], qv[10], qv[11]);
            o.w = (int)pack4(qv[12], qv[13], qv[14], qv[15]);
            *reinterpret_cast<int4*>(p.q + (int64_t)row * p.K + (int64_t)ci * 16) = o;
          }
        }
      }
    }
  }
}

// Paired-chunk per-token int8 kernel (the activation hot path).  Each thread
// owns chunks t and t + TPR of its row and keeps element j of both in one
// float2, so the butterflies, the normalisation and the quantiser issue as
// packed f32x2 instructions (two independent IEEE float32 operations per
// instruction, each rounded exactly like its scalar form).
__device__ __forceinline__ float2 f2_sub(float2 a, float2 b) {
  return f2_fma(b, make_float2(-1.0f, -1.0f), a);  // RN(a - b)
}
__device__ __forceinline__ void h4_regular2(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 m2 = make_float2(-2.0f, -2.0f);
  const float2 s = f2_add(f2_add(a0, a1), f2_add(a2, a3));
  const float2 y0 = f2_fma(a3, m2, s);  // RN(S - 2 a3); 2a is exact
  const float2 y1 = f2_fma(a2, m2, s);
  const float2 y2 = f2_fma(a1, m2, s);
  const float2 y3 = f2_fma(a0, m2, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}
__device__ __forceinline__ void h2_sylvester2(float2& a0, float2& a1) {
  const float2 y0 = f2_add(a0, a1);
  const float2 y1 = f2_sub(a0, a1);
  a0 = y0; a1 = y1;
}
template <int KIND, int N>
__device__ __forceinline__ void xform_regs2(float2* v) {
  if constexpr (KIND == ROT_REGULAR) {
    static_assert(N == 4 || N == 16, "regular Hadamard digits are base 4");
#pragma unroll
    for (int stride = 1; stride < N; stride *= 4)
#pragma unroll
      for (int base = 0; base < N; base += 4 * stride)
#pragma unroll
        for (int o = 0; o < stride; ++o)
          h4_regular2(v[base + o], v[base + o + stride], v[base + o + 2 * stride], v[base + o + 3 * stride]);
  } else if constexpr (KIND == ROT_SYLVESTER) {
#pragma unroll
    for (int stride = 1; stride < N; stride *= 2)
#pragma unroll
      for (int base = 0; base < N; base += 2 * stride)
#pragma unroll
        for (int o = 0; o < stride; ++o) h2_sylvester2(v[base + o], v[base + o + stride]);
  }
}

// One 16-element chunk held as 8 float2 of adjacent elements (2i, 2i+1).
// The within-chunk transform: the stride-1 digit inside each pair (scalar),
// the higher digits on whole pairs (packed); same float32 expressions and
// order as xform_regs<KIND, 16>.
template <int KIND>
__device__ __forceinline__ void xform16_x2(float2 (&v)[8]) {
  if constexpr (KIND == ROT_SYLVESTER) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = v[i].x, b = v[i].y;
      v[i] = make_float2(__fadd_rn(a, b), __fsub_rn(a, b));
    }
#pragma unroll
    for (int ps = 1; ps < 8; ps *= 2)
#pragma unroll
      for (int base = 0; base < 8; base += 2 * ps)
#pragma unroll
        for (int o = 0; o < ps; ++o) h2_sylvester2(v[base + o], v[base + o + ps]);
  } else if constexpr (KIND == ROT_REGULAR) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a0 = v[2 * q].x, a1 = v[2 * q].y, a2 = v[2 * q + 1].x, a3 = v[2 * q + 1].y;
      h4_regular(a0, a1, a2, a3);
      v[2 * q] = make_float2(a0, a1);
      v[2 * q + 1] = make_float2(a2, a3);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) h4_regular2(v[j], v[j + 2], v[j + 4], v[j + 6]);
  }
}

template <int DT>
__device__ __forceinline__ void unpack_raw2(const RawChunk<DT>& r, float2 (&v)[8]) {
  if constexpr (DT == DT_F32) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = make_float2(__uint_as_float(r.w[2 * i]), __uint_as_float(r.w[2 * i + 1]));
  } else if constexpr (DT == DT_BF16) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = make_float2(__uint_as_float(r.w[i] << 16), __uint_as_float(r.w[i] & 0xFFFF0000u));
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __half22float2(*reinterpret_cast<const __half2*>(&r.w[i]));
  }
}

// max of three floats, NaN if any is NaN (sm_100 three-input form).
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Device error word of the row kernels (bit 1: a bulk-copy wait timed out);
// one copy per translation unit, read through rowquant.cu.
static __device__ uint32_t g_rq_error_bits = 0;
// Wait limit in nanoseconds (qlin_set_wait_limit; 2 s by default).
static __device__ uint64_t g_rq_wait_limit_ns = 2000000000ull;

__device__ __forceinline__ bool rq_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_rq_wait_limit_ns);
  const uint64_t t0 = globaltimer_ns();
  uint32_t iter = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++iter & 63u) == 0 && globaltimer_ns() - t0 > limit) {
      atomicOr(&g_rq_error_bits, 2u);
      return false;
    }
  }
}

// Round both halves to the dtype DT (RN-even) and widen back to float.
template <int DT>
__device__ __forceinline__ float2 round2(float2 v) {
  if constexpr (DT == DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    const uint32_t u = *reinterpret_cast<uint32_t*>(&h);
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
  } else if constexpr (DT == DT_F16) {
    return __half22float2(__floats2half2_rn(v.x, v.y));
  } else {
    return v;
  }
}

// 16 elements [16*ci, 16*ci + 16) of a DT vector (16-byte aligned), as pairs.
template <int DT>
__device__ __forceinline__ void load_chunk2(const void* base, int ci, float2 (&v)[8]) {
  RawChunk<DT> raw;
  load_raw<DT>(base, (int64_t)ci * 16, raw);
  unpack_raw2<DT>(raw, v);
}

// Sum of one value per thread over the tpr threads of a row, in a fixed
// order (shuffle tree, then the row's warps in index order); one CTA
// barrier.  buf: [32 rows][17] floats, not touched again before the next
// barrier of the caller.
__device__ __forceinline__ float row_sum(float x, float (*buf)[17], int lane, int warp_in_row, int nw) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, o));
  if (lane == 0) buf[threadIdx.y][warp_in_row] = x;
  __syncthreads();
  float t = buf[threadIdx.y][0];
  for (int w = 1; w < nw; ++w) t = __fadd_rn(t, buf[threadIdx.y][w]);
  return t;
}

// Per-token int8 quantisation of activations (optionally ConvRot-rotated).
// Rows stream through a ring of `stages` shared-memory slots filled by 1-D
// bulk copies (one thread issues them, completion counted on an mbarrier per
// slot), so several rows per CTA are in flight without costing registers.
// Each thread owns CHUNKS 16-element chunks of its row (chunk t + i*TPR),
// each kept as 8 float2 of adjacent elements: the packed float32x2 math, the
// 128-bit shared-memory transposes and the pair-wise bf16 rounding use
// register pairs directly; per-row work (reduction, scale) is shared by
// 16*CHUNKS elements.  The per-row CTA barrier (absmax exchange) also
// releases the row's slot for the next bulk copy.
//
// Dynamic shared memory: [stages x slot_bytes ring][warps x 512 floats
// transpose buffers (rotations with R > 1)][stages mbarriers].
//
// FUSED: the row norm and the modulation of a DiT block run on the row in
// registers before the rotation (two extra CTA barriers per row for the
// layer norm's mean and variance, one for the RMS norm); or (p.situ) the
// SiTU activation of a [hidden | gate] source row, whose ring slot holds
// both halves.
template <int DT, int KIND, int R, int CHUNKS, bool FUSED = false>
__global__ void __launch_bounds__(512) rowquant_x2_kernel(RowQuantParams p, int stages, int slot_bytes) {
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ float red[2][32][17];  // [iteration parity][row][warp]: <= 512 threads, so <= 16 warps per row
  constexpr int EB = DT == DT_F32 ? 4 : 2;  // element bytes
  constexpr bool STAGED = KIND != ROT_NONE && R > 1;

  const int tpr = blockDim.x;
  const int rpc = blockDim.y;
  const int t = threadIdx.x;
  const int tid = threadIdx.y * tpr + t;
  const int lane = t & 31;
  const int warp_in_row = t >> 5;
  const int nchunks = p.K >> 4;
  const int nwarps = (tpr >> 5) * rpc;
  const int warp_lin = threadIdx.y * (tpr >> 5) + warp_in_row;
  const int row_bytes = p.K * EB;
  const int src_bytes = (FUSED && p.situ) ? 2 * row_bytes : row_bytes;  // per ring row
  uint8_t* ring = dsm;
  float* wbuf = reinterpret_cast<float*>(dsm + (size_t)stages * slot_bytes) + warp_lin * 512;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + (size_t)stages * slot_bytes +
                                               (STAGED ? (size_t)nwarps * 512 * sizeof(float) : 0));
  (void)wbuf;

  constexpr int J = 16 / R;
  constexpr int J2 = J < 4 ? J : 4;
  constexpr int NQ = J / J2;
  int nat[4];
  int s2[R > 1 ? R : 1][NQ];
  if constexpr (STAGED) {
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) nat[q4] = swz<R>(lane * 16 + 4 * q4);
    const int g0 = (lane / R) * (16 * R);
    const int rp = lane % R;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int q = 0; q < NQ; ++q) s2[r][q] = swz<R>(g0 + 16 * r + rp * J + q * J2);
  }
  const float2 c2 = make_float2(p.rot_c, p.rot_c);

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();  // before the first global access (launched with PDL)
  pdl_launch_dependents();

  // fill slot s with the rows of iteration `it` (thread 0 only)
  const bool two_src = p.x2 != nullptr;
  const bool dense = !two_src && (int64_t)p.ldx * EB == src_bytes;
  const int bytes1 = two_src ? p.k1 * EB : src_bytes;  // 16-byte multiple (checked by the host)
  auto issue = [&](int it, int s) {
    const int64_t f = ((int64_t)blockIdx.x + (int64_t)it * gridDim.x) * rpc;
    if (f >= p.M) return;
    const int nrows = (int)min((int64_t)rpc, (int64_t)p.M - f);
    mbar_arrive_expect_tx(&full[s], (uint32_t)(nrows * src_bytes));
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.x);
    uint8_t* dst = ring + (size_t)s * slot_bytes;
    if (dense) {
      bulk_load(dst, src + f * src_bytes, (uint32_t)(nrows * src_bytes), &full[s]);
    } else {
      for (int r = 0; r < nrows; ++r) {
        bulk_load(dst + (size_t)r * src_bytes, src + (f + r) * (int64_t)p.ldx * EB, (uint32_t)bytes1, &full[s]);
        if (two_src)
          bulk_load(dst + (size_t)r * src_bytes + bytes1,
                    reinterpret_cast<const uint8_t*>(p.x2) + (f + r) * (int64_t)p.ldx2 * EB,
                    (uint32_t)(src_bytes - bytes1), &full[s]);
      }
    }
  };
  if (tid == 0)
    for (int s = 0; s < stages; ++s) issue(s, s);

  int s = 0;
  uint32_t parity = 0;
  for (int it = 0;; ++it) {
    const int64_t first = ((int64_t)blockIdx.x + (int64_t)it * gridDim.x) * rpc;
    if (first >= p.M) break;
    const bool ok = rq_wait_bounded(&full[s], parity);
    const int64_t row = first + threadIdx.y;
    const bool row_ok = row < p.M && ok;
    const uint8_t* rsrc = ring + (size_t)s * slot_bytes + (size_t)threadIdx.y * src_bytes;
    float2 v[CHUNKS][8];
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const int ci = t + i * tpr;
      if (row_ok && ci < nchunks) {
        RawChunk<DT> raw;
        const uint4* q = reinterpret_cast<const uint4*>(rsrc + (size_t)ci * 16 * EB);
#pragma unroll
        for (int k = 0; k < RawChunk<DT>::WORDS / 4; ++k) {
          const uint4 w = q[k];
          raw.w[4 * k] = w.x; raw.w[4 * k + 1] = w.y; raw.w[4 * k + 2] = w.z; raw.w[4 * k + 3] = w.w;
        }
        unpack_raw2<DT>(raw, v[i]);
        if constexpr (FUSED) {
          if (p.situ) {  // v holds the hidden chunk; its gate chunk sits K elements on
            const uint4* qg = reinterpret_cast<const uint4*>(rsrc + row_bytes + (size_t)ci * 16 * EB);
#pragma unroll
            for (int k = 0; k < RawChunk<DT>::WORDS / 4; ++k) {
              const uint4 w = qg[k];
              raw.w[4 * k] = w.x; raw.w[4 * k + 1] = w.y; raw.w[4 * k + 2] = w.z; raw.w[4 * k + 3] = w.w;
            }
            float2 g[8];
            unpack_raw2<DT>(raw, g);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              v[i][j] = round2<DT>(make_float2(situ_f(v[i][j].x, g[j].x), situ_f(v[i][j].y, g[j].y)));
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = make_float2(0.0f, 0.0f);
      }
    }

    if constexpr (FUSED) {
      // ---- row norm + modulation, in the input dtype's rounding steps ----
      __shared__ float nred[2][32][17];
      const int nw = tpr >> 5;
      if (p.norm_kind != NORM_NONE) {
        const bool layer = p.norm_kind == NORM_LAYER;
        float2 a2 = make_float2(0.0f, 0.0f);  // padding chunks hold zeros
#pragma unroll
        for (int i = 0; i < CHUNKS; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) a2 = layer ? f2_add(a2, v[i][j]) : f2_fma(v[i][j], v[i][j], a2);
        const float m1 = __fdiv_rn(row_sum(__fadd_rn(a2.x, a2.y), nred[0], lane, warp_in_row, nw), (float)p.K);
        if (layer) {
          const float2 mean2 = make_float2(m1, m1);
          float2 b2 = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int i = 0; i < CHUNKS; ++i) {
            if (t + i * tpr >= nchunks) continue;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float2 d = f2_sub(v[i][j], mean2);
              b2 = f2_fma(d, d, b2);
            }
          }
          const float var = __fdiv_rn(row_sum(__fadd_rn(b2.x, b2.y), nred[1], lane, warp_in_row, nw), (float)p.K);
          const float rstd = __frsqrt_rn(__fadd_rn(var, p.eps));
          const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
          for (int i = 0; i < CHUNKS; ++i) {
            const bool pad = t + i * tpr >= nchunks;  // padding chunks stay zero (absmax)
#pragma unroll
            for (int j = 0; j < 8; ++j)
              v[i][j] = pad ? make_float2(0.0f, 0.0f) : round2<DT>(f2_mul(f2_sub(v[i][j], mean2), r2));
          }
        } else {
          // dt((x * rstd) * w): one rounding, as torch's rms_norm
          const float rstd = __frsqrt_rn(__fadd_rn(m1, p.eps));
          const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
          for (int i = 0; i < CHUNKS; ++i) {
            const int ci = t + i * tpr;
            if (p.norm_w != nullptr && ci < nchunks) {
              float2 w[8];
              load_chunk2<DT>(p.norm_w, ci, w);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i][j] = round2<DT>(f2_mul(f2_mul(v[i][j], r2), w[j]));
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) v[i][j] = round2<DT>(f2_mul(v[i][j], r2));
            }
          }
        }
      }
      if (row_ok && (p.mod_mul != nullptr || p.mod_add != nullptr)) {
        const int64_t smp = row / p.rows_per_sample;
#pragma unroll
        for (int i = 0; i < CHUNKS; ++i) {
          const int ci = t + i * tpr;
          if (ci >= nchunks) continue;
          float2 w[8];
          if (p.mod_mul != nullptr) {
            load_chunk2<DT>(reinterpret_cast<const uint8_t*>(p.mod_mul) + smp * p.mul_ld * EB, ci, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = round2<DT>(f2_mul(v[i][j], w[j]));
          }
          if (p.mod_add != nullptr) {
            load_chunk2<DT>(reinterpret_cast<const uint8_t*>(p.mod_add) + smp * p.add_ld * EB, ci, w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = round2<DT>(f2_add(v[i][j], w[j]));
          }
        }
      }
    }

    if constexpr (KIND != ROT_NONE) {
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        xform16_x2<KIND>(v[i]);
        if constexpr (STAGED) {
          // stage 2: transform over the chunk index within each group of R chunks
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4)
            *reinterpret_cast<float4*>(wbuf + nat[q4]) =
                make_float4(v[i][2 * q4].x, v[i][2 * q4].y, v[i][2 * q4 + 1].x, v[i][2 * q4 + 1].y);
          __syncwarp();
          if constexpr (J >= 2) {
            float2 w[J / 2][R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
#pragma unroll
              for (int q = 0; q < NQ; ++q) {
                if constexpr (J2 == 4) {
                  const float4 f = *reinterpret_cast<const float4*>(wbuf + s2[r][q]);
                  w[2 * q][r] = make_float2(f.x, f.y);
                  w[2 * q + 1][r] = make_float2(f.z, f.w);
                } else {
                  w[0][r] = *reinterpret_cast<const float2*>(wbuf + s2[r][q]);
                }
              }
            }
#pragma unroll
            for (int jj = 0; jj < J / 2; ++jj) xform_regs2<KIND, R>(w[jj]);
            // the chunk stays in this transposed layout (element 2jj + c of
            // run r is v[i][jj * R + r].{x,y}); only its int8 codes go back
            // to the natural order, after the row scale is known
#pragma unroll
            for (int jj = 0; jj < J / 2; ++jj)
#pragma unroll
              for (int r = 0; r < R; ++r) v[i][jj * R + r] = w[jj][r];
          } else {
            float w[R];
#pragma unroll
            for (int r = 0; r < R; ++r) w[r] = wbuf[s2[r][0]];
            xform_regs<KIND, R>(w);
#pragma unroll
            for (int r = 0; r < R; r += 2) v[i][r / 2] = make_float2(w[r], w[r + 1]);
          }
          __syncwarp();  // the gathers are done before the next chunk's stores
        }
        // normalise with the dtype-rounded constant, round to the compute dtype
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[i][j] = f2_mul(v[i][j], c2);
          if constexpr (DT == DT_BF16) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[i][j].x, v[i][j].y);
            const uint32_t u = *reinterpret_cast<uint32_t*>(&h);
            v[i][j] = make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
          } else if constexpr (DT == DT_F16) {
            v[i][j] = __half22float2(__floats2half2_rn(v[i][j].x, v[i][j].y));
          }
        }
      }
    }

    // per-row absmax (NaN-propagating); the CTA barrier also frees slot s
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmax3_nan(amax, fabsf(v[i][j].x), fabsf(v[i][j].y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmax_nan(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const int nw = tpr >> 5;
    float (*rb)[17] = red[it & 1];
    if (lane == 0) rb[threadIdx.y][warp_in_row] = amax;
    if (__syncthreads_or(!ok)) break;  // a bulk copy never arrived: leave together
    if (tid == 0) {
      fence_proxy_async_smem();  // this iteration's reads of slot s before the next copy into it
      issue(it + stages, s);
    }
    if (++s == stages) { s = 0; parity ^= 1; }
    amax = rb[threadIdx.y][0];
    for (int w2 = 1; w2 < nw; ++w2) amax = fmax_nan(amax, rb[threadIdx.y][w2]);
    if (!row_ok) continue;
    int8_t* qrow = p.q + row * p.K;
    if (!(amax < __uint_as_float(0x7F800000u))) {
      // Inf or NaN in the row: scale Inf / NaN and every code 0 (torch's result)
      if (t == 0) p.scale[row] = amax;
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        const int ci = t + i * tpr;
        if (ci < nchunks) *reinterpret_cast<int4*>(qrow + (int64_t)ci * 16) = make_int4(0, 0, 0, 0);
      }
      continue;
    }
    const float s_row = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);  // (absmax.float()/127).clamp(1e-30)
    const float inv = __frcp_rn(s_row);                          // 1.0 / scale
    if (t == 0) p.scale[row] = s_row;
    // |v| <= absmax: the round-half-even code of v * (1/scale) is already in
    // [-127, 127]; the low byte of y + 1.5*2^23 is its two's complement.  The
    // product is rounded before the add (torch rounds x * (1/s), then to an
    // integer); the add is an FMA with a run-time 1.0 so that the assembler
    // cannot fuse it with the packed multiply (it did fuse a plain packed add).
    const float2 inv2 = make_float2(inv, inv);
    const float2 one2 = make_float2(p.one, p.one);
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    if constexpr (STAGED) {
      // Run r of this lane's transposed chunk is the J elements at offset
      // g0 + 16 r + rp J of the warp's 512-element span (the lane's rotation
      // group starts at g0).  Their codes are stored there in a byte image
      // of the span (16-byte segment index XOR-ed with the 128-byte row, so
      // a store instruction and the 16-byte natural reads hit distinct
      // banks); each lane then reads its own natural chunk back.
      uint8_t* cb = reinterpret_cast<uint8_t*>(wbuf);
      const int base = (lane / R) * (16 * R) + (lane % R) * J;
      auto cswz = [](int a) { return a ^ (((a >> 7) & 7) << 4); };
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        int c[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 y = f2_fma(f2_mul(v[i][j], inv2), one2, magic);
          c[2 * j] = (int)__float_as_uint(y.x);
          c[2 * j + 1] = (int)__float_as_uint(y.y);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          uint8_t* d = cb + cswz(base + 16 * r);
          if constexpr (J == 1) {
            *d = (uint8_t)c[r];
          } else if constexpr (J == 2) {
            *reinterpret_cast<uint16_t*>(d) = (uint16_t)__byte_perm((uint32_t)c[2 * r], (uint32_t)c[2 * r + 1], 0x0040);
          } else if constexpr (J == 4) {
            *reinterpret_cast<uint32_t*>(d) = pack4(c[2 * r], c[2 * r + 1], c[2 * (R + r)], c[2 * (R + r) + 1]);
          } else {
            static_assert(J == 8, "runs of 1, 2, 4 or 8 elements");
            *reinterpret_cast<uint2*>(d) =
                make_uint2(pack4(c[2 * r], c[2 * r + 1], c[2 * (R + r)], c[2 * (R + r) + 1]),
                           pack4(c[2 * (2 * R + r)], c[2 * (2 * R + r) + 1], c[2 * (3 * R + r)], c[2 * (3 * R + r) + 1]));
          }
        }
        __syncwarp();
        const uint4 o = *reinterpret_cast<const uint4*>(cb + cswz(16 * lane));
        __syncwarp();  // read before the next chunk's (or row's) stores
        const int ci = t + i * tpr;
        if (ci < nchunks) *reinterpret_cast<uint4*>(qrow + (int64_t)ci * 16) = o;
      }
    } else {
#pragma unroll
      for (int i = 0; i < CHUNKS; ++i) {
        const int ci = t + i * tpr;
        if (ci >= nchunks) continue;
        uint32_t u[16];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float2 y = f2_fma(f2_mul(v[i][j], inv2), one2, magic);
          u[2 * j] = __float_as_uint(y.x);
          u[2 * j + 1] = __float_as_uint(y.y);
        }
        int4 o;
        o.x = (int)pack4((int)u[0], (int)u[1], (int)u[2], (int)u[3]);
        o.y = (int)pack4((int)u[4], (int)u[5], (int)u[6], (int)u[7]);
        o.z = (int)pack4((int)u[8], (int)u[9], (int)u[10], (int)u[11]);
        o.w = (int)pack4((int)u[12], (int)u[13], (int)u[14], (int)u[15]);
        *reinterpret_cast<int4*>(qrow + (int64_t)ci * 16) = o;
      }
    }
  }
}

// Generic fallback for rows that are not 16-element aligned (no rotation):
// one CTA per row, strided scalar loop, two passes over the row.
template <int DT_IN, int MODE>
__global__ void __launch_bounds__(256) rowquant_generic_kernel(RowQuantParams p) {
  using EQ = Elem<DT_IN>;
  using T = typename Elem<DT_IN>::T;
  __shared__ float red[8];
  const int row = blockIdx.x;
  const T* x = reinterpret_cast<const T*>(p.x) + (int64_t)row * p.ldx;
  float a = 0.0f;
  for (int k = threadIdx.x; k < p.K; k += blockDim.x) a = fmaxf(a, fabsf(EQ::to_f(x[k])));
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  a = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) a = fmaxf(a, red[w]);
  float s, inv = 0.0f;
  if constexpr (MODE == MODE_INT8) {
    s = fmaxf(__fdiv_rn(a, 127.0f), 1e-30f);
    inv = __frcp_rn(s);
  } else {
    s = EQ::round(__fdiv_rn(fmaxf(a, p.clamp_min), 7.0f));
  }
  if (threadIdx.x == 0) p.scale[row] = s;
  for (int k = threadIdx.x; k < p.K; k += blockDim.x) {
    const float xv = EQ::to_f(x[k]);
    float y;
    if constexpr (MODE == MODE_INT8) {
      y = fminf(fmaxf(__fmul_rn(xv, inv), -128.0f), 127.0f);
    } else {
      y = EQ::round(__fdiv_rn(xv, s));
      y = (y != y) ? 0.0f : fminf(fmaxf(y, -7.0f), 7.0f);
    }
    p.q[(int64_t)row * p.K + k] = (int8_t)rint_to_int(y);
  }
}

}  // namespace qlin
