// Per-token int8 quantisation of 16-bit activations, fused with the ConvRot
// rotation: the activation hot path of the W8A8 linear.
//
// Each thread owns one 128-element strip of a row and keeps it in registers
// from the single HBM read to the single HBM write:
//   1. sixteen 16-byte shared-memory reads of the strip (rows arrive by bulk
//      copy), widened to float32 pairs;
//   2. the Hadamard transform of the strip's rotation groups entirely in
//      registers (Sylvester 128: all seven butterfly stages; regular 256:
//      three base-4 digits in registers, the fourth across a lane pair);
//   3. times the normalisation constant, rounded to the dtype and packed two
//      per register; absmax on the packed pairs (NaN-propagating);
//   4. one shared-memory atomicMax per strip and one CTA barrier give the
//      row's absmax (non-negative float32 bit patterns order as integers;
//      every NaN pattern sorts above infinity);
//   5. scale, codes with the reference's rounding sequence, stored from
//      registers.
// No shared-memory transposes: the only cross-thread exchange of a rotation
// is the regular-256 top digit (one shuffle per element).  A CTA holds whole
// rows, at most 128 threads.
//
// The float32 expressions and their order are those of the other row kernels
// and of the oracle: Sylvester stages a0 + a1, a0 - a1 from the least
// significant index bit up; regular digits S = (a0 + a1) + (a2 + a3),
// y_k = S - 2 a_{3-k}; then times the dtype-rounded constant, rounded to the
// dtype; scale = max(absmax / 127, 1e-30), codes = rne(v * RN(1 / scale)).
#pragma once

#include "rowquant.cuh"  // rq_wait_bounded, the row kernels' error word

namespace qlin {

constexpr int STRIP = 128;  // elements per thread

// Two 16-bit values (lo = x) rounded from a float pair.
template <int DT>
__device__ __forceinline__ uint32_t strip_pack_rn(float2 v) {
  if constexpr (DT == DT_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(v.x, v.y);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <int DT>
__device__ __forceinline__ float2 strip_unpack(uint32_t w) {
  if constexpr (DT == DT_BF16) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
}
// Per 16-bit half: max(|a|, |b|), NaN if either is NaN (the sign bits of the
// result are sign(a) ^ sign(b) and are discarded by the caller).
template <int DT>
__device__ __forceinline__ uint32_t strip_absmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (DT == DT_BF16) {
    asm("max.NaN.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  } else {
    asm("max.NaN.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  }
  return r;
}

__device__ __forceinline__ void st256(void* p, const uint32_t (&r)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r[0]), "r"(r[1]), "r"(r[2]),
               "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

// Hadamard digits of the strip held as NP float pairs (elements 2p, 2p + 1),
// over the strip-local index bits below log2(G) (G <= 2 NP; G = 64 is also
// the in-register part of a regular 256 group and of a Sylvester 128 group
// split over a lane pair).
template <int KIND, int G, int NP>
__device__ __forceinline__ void strip_xform(float2 (&v)[NP]) {
  if constexpr (KIND == ROT_SYLVESTER) {
    static_assert(G == 32 || G == 64 || G == 128, "Sylvester sizes 32, 64 (half group) and 128");
    static_assert(G <= 2 * NP, "the digits lie inside the strip");
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const float a = v[p].x, b = v[p].y;
      v[p] = make_float2(__fadd_rn(a, b), __fsub_rn(a, b));
    }
#pragma unroll
    for (int ps = 1; ps < G / 2; ps *= 2)
#pragma unroll
      for (int base = 0; base < NP; base += 2 * ps)
#pragma unroll
        for (int o = 0; o < ps; ++o) {
          const float2 a0 = v[base + o], a1 = v[base + o + ps];
          v[base + o] = f2_add(a0, a1);
          v[base + o + ps] = f2_fma(a1, make_float2(-1.0f, -1.0f), a0);  // RN(a0 - a1)
        }
  } else if constexpr (KIND == ROT_REGULAR) {
    static_assert(G == 16 || G == 64, "in-register regular digits cover 16 or 64 elements");
#pragma unroll
    for (int q = 0; q < NP / 2; ++q) {
      float a0 = v[2 * q].x, a1 = v[2 * q].y, a2 = v[2 * q + 1].x, a3 = v[2 * q + 1].y;
      h4_regular(a0, a1, a2, a3);
      v[2 * q] = make_float2(a0, a1);
      v[2 * q + 1] = make_float2(a2, a3);
    }
#pragma unroll
    for (int ps = 2; ps < G / 2; ps *= 4)
#pragma unroll
      for (int base = 0; base < NP; base += 4 * ps)
#pragma unroll
        for (int o = 0; o < ps; ++o) {
          const float2 m2 = make_float2(-2.0f, -2.0f);
          const float2 a0 = v[base + o], a1 = v[base + o + ps], a2 = v[base + o + 2 * ps], a3 = v[base + o + 3 * ps];
          const float2 s = f2_add(f2_add(a0, a1), f2_add(a2, a3));
          v[base + o] = f2_fma(a3, m2, s);
          v[base + o + ps] = f2_fma(a2, m2, s);
          v[base + o + 2 * ps] = f2_fma(a1, m2, s);
          v[base + o + 3 * ps] = f2_fma(a0, m2, s);
        }
  }
}

// Top base-4 digit of a regular 256 group split over a lane pair.  The lane
// with pair bit b holds group elements 64b + u (local u < 64) and
// 128 + 64b + u (local u + 64), i.e. digit values a_b and a_{b+2}; both lanes
// evaluate S = (a0 + a1) + (a2 + a3) with the same operands (the additions
// commute exactly) and y_k = S - 2 a_{3-k} for their own two values.
// `lanes`: the lanes of this warp that exist (a CTA need not fill its last
// warp; lane pairs never straddle it, the strips per row being even).
__device__ __forceinline__ void strip_regular256_top(float2 (&v)[64], unsigned lanes) {
  const float2 m2 = make_float2(-2.0f, -2.0f);
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    const float2 lo = v[p], hi = v[p + 32];
    const float2 plo = make_float2(__shfl_xor_sync(lanes, lo.x, 1), __shfl_xor_sync(lanes, lo.y, 1));
    const float2 phi = make_float2(__shfl_xor_sync(lanes, hi.x, 1), __shfl_xor_sync(lanes, hi.y, 1));
    const float2 s = f2_add(f2_add(lo, plo), f2_add(hi, phi));
    v[p] = f2_fma(phi, m2, s);       // y_b     = S - 2 a_{3-b}
    v[p + 32] = f2_fma(plo, m2, s);  // y_{b+2} = S - 2 a_{1-b}
  }
}

// Top (seventh) Sylvester stage of a 128 group split over a lane pair: the
// lane with pair bit b holds group elements 64b + u; y_u = RN(a_u + a_{64+u})
// on the even lane and y_{64+u} = RN(a_u - a_{64+u}) on the odd one, both as
// RN(sgn * mine + partner) with sgn = +1 / -1 (the product is exact).
__device__ __forceinline__ void strip_sylvester128_top(float2 (&v)[32], unsigned lanes, bool odd) {
  const float2 sg = odd ? make_float2(-1.0f, -1.0f) : make_float2(1.0f, 1.0f);
#pragma unroll
  for (int p = 0; p < 32; ++p) {
    const float2 pv = make_float2(__shfl_xor_sync(lanes, v[p].x, 1), __shfl_xor_sync(lanes, v[p].y, 1));
    v[p] = f2_fma(v[p], sg, pv);
  }
}

// x [M, K] (row stride ldx elements), or with x2 the concatenated rows
// [x[r, 0:k1] | x2[r, 0:K-k1]] (k1 and K - k1 multiples of 8, row strides ldx
// and ldx2); K a multiple of 128 with K / SW <= 128; q [M, K] int8 (32-byte aligned), scale [M].  rot_c: the dtype-rounded
// +-entry of the normalised Hadamard; one: 1.0f at run time (the
// quantiser's add is an FMA by it, which the assembler cannot contract with
// the preceding multiply).
//
// SW: elements per thread, 128, or 64 for Sylvester 128 (a group split over
// a lane pair: six stages in registers, the seventh by one shuffle per
// element; half the registers, so about twice the warps per SM).
//
// Persistent CTAs of `rows` whole rows (blockDim.x = rows * K / SW)
// stream row blocks through a ring of `stages` shared-memory slots filled
// by 1-D bulk copies (one thread issues them; completion counted on an
// mbarrier per slot), so the next blocks' loads are in flight while a block
// is rotated and quantised.  The per-block CTA barrier (row absmax) also
// frees the block's slot for its next copy.
//
// Bank-conflict-free strip reads: lane l reads 16-byte chunk i ^ d of its
// strip into register chunk i (d = l & 7; for a group split over a lane
// pair the pair's shared d = (l >> 1) & 7, so the relabelling is one XOR of
// the group index), so a warp's 16-byte reads cover all eight bank
// columns.  Relabelling the inputs of a Hadamard transform by an XOR of the
// index is undone exactly on the outputs:
//  * Sylvester: H P = S H with S diagonal +-1, so output k keeps its place
//    and flips sign when popcount(D & k) is odd (every butterfly node is the
//    correspondingly signed node of the unpermuted transform, the additions
//    commute and RN is sign-symmetric); bits of D above the group permute
//    whole groups.  The sign is folded into the normalisation constant.
//  * regular H4 digits: S is the same sum and y_k = S - 2 a_{3-k} lands at
//    k ^ delta: outputs are permuted by the same XOR.
//  * no rotation: a plain permutation.
// Codes of register chunk i are stored at chunk (i ^ d) -- except
// Sylvester 128, whose outputs keep their place: natural order, 256-bit
// stores.
template <int DT, int KIND, int G, int SW = 128>
__global__ void __launch_bounds__(128, SW == 64 ? 5 : 3)
    rowquant_strip_kernel(const void* __restrict__ x, int64_t ldx, const void* __restrict__ x2, int64_t ldx2, int k1,
                          int M, int K, int rows, int stages, int slot_bytes, float rot_c, float one,
                          int8_t* __restrict__ q, float* __restrict__ scale) {
  static_assert(DT == DT_BF16 || DT == DT_F16, "16-bit activations");
  static_assert(SW == 128 || (SW == 64 && KIND == ROT_SYLVESTER && G == 128), "half strips: Sylvester 128");
  constexpr bool PAIR = KIND == ROT_REGULAR && G == 256;  // a group spans two strips
  constexpr bool HALF = SW == 64;                          // a Sylvester 128 group spans two strips
  constexpr bool NATURAL = KIND == ROT_SYLVESTER && G == 128;  // outputs keep their place
  constexpr int NC = SW / 8;  // 16-byte chunks per strip
  constexpr int NP = SW / 2;  // float pairs per strip
  extern __shared__ __align__(128) uint8_t dsm[];
  __shared__ uint32_t s_amax[3][128];
  __shared__ uint64_t full[4];
  const int T = K / SW;  // strips per row
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int r = tid / T;
  const int j = tid - r * T;
  const int nblocks = (M + rows - 1) / rows;
  const int row_bytes = K * 2;
  const bool dense = x2 == nullptr && ldx == (int64_t)K;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < 3 * 128; i += blockDim.x) (&s_amax[0][0])[i] = 0u;
  __syncthreads();
  pdl_wait();  // the previous kernel's rows and codes buffers are settled
  pdl_launch_dependents();

  auto issue = [&](int it, int s) {  // thread 0: row block of iteration `it` into slot s
    const int64_t b = (int64_t)blockIdx.x + (int64_t)it * gridDim.x;
    if (b >= nblocks) return;
    const int64_t f = b * rows;
    const int n = (int)min((int64_t)rows, (int64_t)M - f);
    mbar_arrive_expect_tx(&full[s], (uint32_t)(n * row_bytes));
    const uint8_t* src = reinterpret_cast<const uint8_t*>(x);
    uint8_t* dst = dsm + (size_t)s * slot_bytes;
    if (dense) {
      bulk_load(dst, src + f * row_bytes, (uint32_t)(n * row_bytes), &full[s]);
    } else if (x2 != nullptr) {  // row = [x[r, 0:k1] | x2[r, 0:K-k1]]
      const uint8_t* src2 = reinterpret_cast<const uint8_t*>(x2);
      const int b1 = k1 * 2;
      for (int k = 0; k < n; ++k) {
        bulk_load(dst + (size_t)k * row_bytes, src + (f + k) * ldx * 2, (uint32_t)b1, &full[s]);
        bulk_load(dst + (size_t)k * row_bytes + b1, src2 + (f + k) * ldx2 * 2, (uint32_t)(row_bytes - b1), &full[s]);
      }
    } else {
      for (int k = 0; k < n; ++k) bulk_load(dst + (size_t)k * row_bytes, src + (f + k) * ldx * 2, (uint32_t)row_bytes, &full[s]);
    }
  };
  if (tid == 0)
    for (int s = 0; s < stages; ++s) issue(s, s);

  const int d = (PAIR || HALF) ? (lane >> 1) & 7 : lane & 7;
  // strip-local chunk c (8 elements) lives at column col(c) of the row:
  // contiguous, or (PAIR) two 64-element halves of the group, 128 apart
  const int c_lo = PAIR ? (j >> 1) * 256 + (j & 1) * 64 : j * SW;
  const int c_hi = PAIR ? c_lo + 128 : c_lo + 64;
  auto chunk_col = [&](int c) { return c < 8 ? c_lo + 8 * c : c_hi + 8 * (c - 8); };

  int s = 0;
  uint32_t parity = 0;
  for (int it = 0;; ++it) {
    const int64_t b = (int64_t)blockIdx.x + (int64_t)it * gridDim.x;
    if (b >= nblocks) break;
    const bool ok = rq_wait_bounded(&full[s], parity);
    const int64_t row = b * rows + r;
    const bool live = row < M && ok;
    const uint8_t* slot = dsm + (size_t)s * slot_bytes + (size_t)r * row_bytes;

    float2 v[NP];
    uint32_t pk[NP];
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = i ^ d;  // i and c share bit 3 (the 64-element half)
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      if (live) w = *reinterpret_cast<const uint4*>(slot + 2 * chunk_col(c));
      pk[4 * i] = w.x; pk[4 * i + 1] = w.y; pk[4 * i + 2] = w.z; pk[4 * i + 3] = w.w;
    }
    if constexpr (KIND != ROT_NONE) {
#pragma unroll
      for (int p = 0; p < NP; ++p) v[p] = strip_unpack<DT>(pk[p]);
      if constexpr (PAIR || HALF) {
        strip_xform<KIND, 64>(v);
        const int in_warp = (int)blockDim.x - (tid & ~31);
        const unsigned lanes = in_warp >= 32 ? 0xffffffffu : (1u << in_warp) - 1u;
        if constexpr (PAIR) strip_regular256_top(v, lanes);
        else strip_sylvester128_top(v, lanes, (lane & 1) != 0);
      } else {
        strip_xform<KIND, G>(v);
      }
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        float ci = rot_c;
        if constexpr (KIND == ROT_SYLVESTER) {
          constexpr int GC = G / 8;  // chunks per group
          if (__popc(d & i & (GC - 1)) & 1) ci = -rot_c;
        }
        const float2 c2 = make_float2(ci, ci);
#pragma unroll
        for (int k = 0; k < 4; ++k) pk[4 * i + k] = strip_pack_rn<DT>(f2_mul(v[4 * i + k], c2));
      }
    }

    // absmax of the strip on packed pairs, then of the row
    uint32_t m = pk[0];
#pragma unroll
    for (int p = 1; p < NP; ++p) m = strip_absmax2<DT>(m, pk[p]);
    float a0, a1;
    if constexpr (DT == DT_BF16) {
      a0 = __uint_as_float((m << 16) & 0x7FFFFFFFu);
      a1 = __uint_as_float(m & 0x7FFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&m));
      a0 = fabsf(f.x);
      a1 = fabsf(f.y);
    }
    const uint32_t ab = max(__float_as_uint(a0), __float_as_uint(a1));  // NaN patterns sort highest
    uint32_t* am = s_amax[it % 3];
    if (live) atomicMax(&am[r], ab);
    if (__syncthreads_or(!ok)) break;  // a bulk copy never arrived: leave together
    if (tid == 0) {
      fence_proxy_async_smem();  // this block's reads of slot s before the next copy into it
      issue(it + stages, s);
    }
    if (tid < rows) s_amax[(it + 2) % 3][tid] = 0u;  // last read in iteration it - 1
    if (++s == stages) { s = 0; parity ^= 1; }
    if (!live) continue;
    const float amax = __uint_as_float(am[r]);

    int8_t* qr = q + row * (int64_t)K;
    if (!(amax < __uint_as_float(0x7F800000u))) {
      // Inf or NaN in the row: scale Inf / NaN and every code 0 (torch's result)
      if (j == 0) scale[row] = amax;
#pragma unroll
      for (int i = 0; i < NC; ++i) *reinterpret_cast<uint2*>(qr + chunk_col(i)) = make_uint2(0u, 0u);
      continue;
    }
    const float s_row = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);  // (absmax.float() / 127).clamp(1e-30)
    const float inv = __frcp_rn(s_row);                          // 1.0 / scale
    if (j == 0) scale[row] = s_row;
    // |v| <= absmax: the round-half-even code of v * (1/scale) is already in
    // [-127, 127] and is the low byte of RN(v * inv) + 1.5 * 2^23.
    const float2 inv2 = make_float2(inv, inv);
    const float2 one2 = make_float2(one, one);
    const float2 magic = make_float2(12582912.0f, 12582912.0f);
    uint32_t cw[NP / 2];  // codes of register chunk i: cw[2i], cw[2i + 1]
#pragma unroll
    for (int w = 0; w < NP / 2; ++w) {
      const float2 ya = f2_fma(f2_mul(strip_unpack<DT>(pk[2 * w]), inv2), one2, magic);
      const float2 yb = f2_fma(f2_mul(strip_unpack<DT>(pk[2 * w + 1]), inv2), one2, magic);
      const uint32_t lo = __byte_perm(__float_as_uint(ya.x), __float_as_uint(ya.y), 0x0040);
      const uint32_t hi = __byte_perm(__float_as_uint(yb.x), __float_as_uint(yb.y), 0x0040);
      cw[w] = __byte_perm(lo, hi, 0x5410);
    }
    if constexpr (NATURAL) {
#pragma unroll
      for (int h = 0; h < SW / 32; ++h) {
        const uint32_t o[8] = {cw[8 * h], cw[8 * h + 1], cw[8 * h + 2], cw[8 * h + 3],
                               cw[8 * h + 4], cw[8 * h + 5], cw[8 * h + 6], cw[8 * h + 7]};
        st256(qr + j * SW + 32 * h, o);
      }
    } else {
      // Sylvester: only XOR bits above the group move outputs; regular and
      // no rotation: the whole XOR
      constexpr int MOVE = KIND == ROT_SYLVESTER ? 7 & ~(G / 8 - 1) : 7;
#pragma unroll
      for (int i = 0; i < NC; ++i)
        *reinterpret_cast<uint2*>(qr + chunk_col(i ^ (d & MOVE))) = make_uint2(cw[2 * i], cw[2 * i + 1]);
    }
  }
}

}  // namespace qlin
