// Group-128 packed-int4-weight GEMMs on the tcgen05 tensor cores:
//
//   W4A8: acc = 0; for g: acc = fmaf(float(P_g[m,n]), ws[n,g], acc)
//         out = dt(dt32(acc * xs[m]) + bias[n])
//   W4A4: acc = 0; for g: acc = fmaf(float(P_g[m,n]), dt32(xs[m,g] * ws[n,g]), acc)
//         out = dt(acc + bias[n])
//
// with P_g the exact int32 dot product over K-group g (128 elements), A int8
// codes [M, K] (int8 per-token for W4A8, int4-range codes for W4A4), W packed
// int4 [N, K/2] (low nibble = even k), ws bf16 [N, K/128].
//
// One K-slab of the pipeline is exactly one scale group, so the MMA writes
// each group's partial into its own TMEM buffer (four, in rotation) and the
// epilogue warps fold it into a float32 accumulator held in registers:
//   warpgroup 0 (64 registers): warp 0 TMA producer (A slab 128x128 int8,
//               swizzled; packed W slab), warp 1 TMEM allocator + MMA issuer
//               (M=128, N=128, K=32 x 4 per group), warps 2-3 idle
//   warpgroups 1-2 (192 registers): epilogue, per group TMEM partial ->
//               float -> fma into a 64-float register accumulator (rows: the
//               warp's TMEM lane quarter, columns: its half of the tile)
//   warpgroup 3 (64 registers): nibble unpack of the W slab into the
//               swizzled int8 layout.
// Registers at launch: 512 threads x 128; after setmaxnreg
// 128 x 64 + 256 x 192 + 128 x 64 = 65536, the launch total.
//
// Two exact transformations keep the epilogue short:
//  * nibbles are unpacked as 16*q (the nibble moved to the high half of the
//    byte: no sign extension), so the MMA produces 16*P_g; the group scales
//    are stored divided by 16, and 16*P * (s/16) == P * s exactly;
//  * each partial buffer is pre-loaded with the bits of 1.5*2^23 and the MMA
//    accumulates on top, so float(16*P) = as_float(bits) - 1.5*2^23 exactly
//    (|16*P| < 2^22), one subtraction instead of an int-to-float conversion.
// No TMA multicast; every pipeline wait is bounded (g_error_bits, abort flag).
#pragma once

#include <type_traits>

#include "gemm_i8.cuh"

namespace qlin {

enum : int { G128_W4A8 = 0, G128_W4A4 = 1 };

struct G128Params {
  int M, N, K;
  const float* a_scale;       // W4A8: [M]; W4A4: [M, K/128]
  const uint16_t* w_gscale;   // bf16 bits [N, K/128]
  const void* bias;           // [N] in the output dtype, or null
  void* out;                  // [M, N]
  int64_t ldo;
};

struct G128Cfg {
  static constexpr int BM = 128, BN = 128, BK = 128;  // BK = scale group
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = BM * BK;             // 16 KB
  static constexpr int B_BYTES = BN * BK;             // 16 KB unpacked
  static constexpr int BP_BYTES = BN * BK / 2;        // 8 KB packed
  static constexpr int NUM_THREADS = 512;  // 4 warpgroups
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES + BP_BYTES) + 256 + 16 + 8 * 2 * 64 * 4 + 16;
  static_assert(3 * STAGES * 8 + 2 * 4 * 8 + 16 + 16 <= 256 + 16 + 16, "barrier block overflows its reserve");
  static constexpr uint32_t TMEM_COLS = 4 * BN;  // G128_NBUF partial buffers
};

constexpr uint32_t kG128Magic = 0x4B400000u;  // bits of 1.5 * 2^23
constexpr int G128_NBUF = 4;                   // TMEM partial buffers (4 x 128 columns)

// 32 lanes x 8 columns of 32-bit TMEM <- 8 registers per thread.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
               : "memory");
}
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 lanes x 16 columns of 32-bit TMEM -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Store 8 consecutive outputs (already rounded to DT) of one row.
template <int DT>
__device__ __forceinline__ void store8(typename Elem<DT>::T* dst, const float (&y)[8], bool vec, int n) {
  if (vec && n >= 8) {
    if constexpr (DT == DT_F32) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (DT == DT_BF16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < n) dst[j] = Elem<DT>::from_f(y[j]);
  }
}

// Group scale of column `col`, group g, as float divided by 16 (exact).
__device__ __forceinline__ float g128_wscale16(const G128Params& p, int G, int col, int g) {
  if (col >= p.N) return 0.0f;
  const uint16_t b = __ldg(p.w_gscale + (int64_t)col * G + g);
  return __uint_as_float((uint32_t)b << 16) * 0.0625f;
}

template <int MODE, int OUT_DT>
__global__ void __launch_bounds__(G128Cfg::NUM_THREADS, 1)
    gemm_g128_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     G128Params p) {
  using Cfg = G128Cfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* sBP = sB + STAGES * Cfg::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sBP + STAGES * Cfg::BP_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;
  uint64_t* pfull = conv + STAGES;           // [G128_NBUF] partial of a group ready
  uint64_t* pempty = pfull + G128_NBUF;      // [G128_NBUF] partial consumed and re-biased
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pempty + G128_NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));
  // s_ws[8 warps][2][64]: group scales / 16 of each epilogue warp's columns

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);
    }
    for (int b = 0; b < G128_NBUF; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + Cfg::BM - 1) / Cfg::BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int G = p.K / Cfg::BK;

  // each role's code sits inside the branch that set its register limit
  if (warp < 4) {
    regs_dec<64>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int g = 0; g < G; ++g) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::BP_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], g * Cfg::BK, mb * Cfg::BM);
          tma_load_2d(sBP + stage * Cfg::BP_BYTES, &tmB, &full[stage], g * (Cfg::BK / 2), nb * BN);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = umma_idesc_i8(Cfg::BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int b = 0;
      uint32_t pph = 0;  // phase of the pempty round (flips when b wraps)
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        for (int g = 0; g < G; ++g) {
          if (!mbar_wait_bounded(&conv[stage], phase, abort_flag) ||
              !mbar_wait_bounded(&pempty[b], pph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_k_sw128(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bdesc = umma_desc_k_sw128(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < Cfg::BK / 32; ++k)  // accumulate onto the 1.5*2^23 bias
            umma_i8(tmem_base + b * BN, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
          umma_commit(&empty[stage]);
          umma_commit(&pfull[b]);
          if (++b == G128_NBUF) { b = 0; pph ^= 1; }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp < 12) {
    regs_inc<192>();
    // ---------------- epilogue ----------------
    using EO = Elem<OUT_DT>;
    const int e = (warp - 4) * 32 + lane;  // 0..255
    const int quarter = warp & 3;          // TMEM lanes 32*quarter.. (warp % 4 rule)
    const int half = (warp - 4) >> 2;      // columns 64*half..
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;

    // bias every partial buffer region this warp owns, then hand all
    // buffers to the MMA (phase 0 of pempty)
#pragma unroll
    for (int b = 0; b < G128_NBUF; ++b)
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) tmem_st_32x32b_x8(tmem_base + b * BN + half * 64 + c8 * 8 + lane_off, kG128Magic);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < G128_NBUF; ++b) mbar_arrive(&pempty[b]);

    // A step is one (tile, group) in issue order.  Each warp stages the 64
    // column scales of its half of the tile in its own shared-memory buffer
    // (double-buffered by step parity, __syncwarp only); every lane loads two
    // of them, five steps ahead, into a 4-slot register ring whose slot index
    // is static (the step loop is unrolled by 4).  W4A4 row scales are loaded
    // four steps ahead the same way.
    struct It {
      int tile, g, mb, nb;
    };
    auto it_at = [&](int tile) {
      It t{tile, 0, 0, 0};
      if (tile < num_tiles) tile_coords(tile, num_m, num_n, t.mb, t.nb);
      return t;
    };
    auto it_adv = [&](It& t) {
      if (++t.g == G) {
        t.g = 0;
        t.tile += gridDim.x;
        if (t.tile < num_tiles) tile_coords(t.tile, num_m, num_n, t.mb, t.nb);
      }
    };
    auto load_ws = [&](const It& t, int j) -> float {  // column half*64 + 32*j + lane
      if (t.tile >= num_tiles) return 0.0f;
      return g128_wscale16(p, G, t.nb * BN + half * 64 + 32 * j + lane, t.g);
    };
    auto load_xs = [&](const It& t) -> float {
      if (t.tile >= num_tiles) return 0.0f;
      const int row2 = t.mb * Cfg::BM + quarter * 32 + lane;
      if (row2 >= p.M) return 0.0f;
      if constexpr (MODE == G128_W4A8) return __ldg(p.a_scale + row2);
      else return __ldg(p.a_scale + (int64_t)row2 * G + t.g);
    };

    float* wbuf = s_ws + (warp - 4) * 128;  // [2][64] floats of this warp
    It cur = it_at(blockIdx.x);
    It la = cur;
    wbuf[lane] = load_ws(la, 0);
    wbuf[32 + lane] = load_ws(la, 1);
    float rw0[4], rw1[4];  // scale of step t in slot t % 4
#pragma unroll
    for (int k = 1; k <= 4; ++k) {
      it_adv(la);
      rw0[k & 3] = load_ws(la, 0);
      rw1[k & 3] = load_ws(la, 1);
    }
    it_adv(la);  // step 5
    It lx = cur;
    float rxs[4];  // W4A4: row scale of step t in slot t % 4
    if constexpr (MODE == G128_W4A4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        rxs[k] = load_xs(lx);
        it_adv(lx);
      }
    }
    float xs_row = 0.0f, xs_next = 0.0f;  // W4A8 row scale: this tile, next tile
    if constexpr (MODE == G128_W4A8) {
      xs_row = load_xs(cur);
      xs_next = load_xs(it_at(cur.tile + (int)gridDim.x));
    }
    __syncwarp();

    float2 acc[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    int b = 0;
    uint32_t pph = 0;  // phase of the pfull round (flips when b wraps)

    // one step; K = step % 4 (static).  Returns false when this CTA is done.
    auto step_fn = [&](auto kc) -> bool {
      constexpr int K = decltype(kc)::value;
      constexpr int K1 = (K + 1) & 3;
      if (cur.tile >= num_tiles) return false;
      const bool ok = mbar_wait_bounded(&pfull[b], pph, abort_flag);
      if (__any_sync(0xffffffffu, !ok || *abort_flag)) return false;
      tc_fence_after();
      uint32_t r[64];
      tmem_ld_32x32b_x32(tmem_base + b * BN + half * 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(tmem_base + b * BN + half * 64 + 32 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      const float* ws_cur = wbuf + (K & 1) * 64;
      float* ws_nxt = wbuf + (K1 & 1) * 64;
      ws_nxt[lane] = rw0[K1];
      ws_nxt[32 + lane] = rw1[K1];
      rw0[K1] = load_ws(la, 0);  // step + 5
      rw1[K1] = load_ws(la, 1);
      it_adv(la);
      float xs_g = 0.0f;
      if constexpr (MODE == G128_W4A4) {
        xs_g = rxs[K];
        rxs[K] = load_xs(lx);  // step + 4
        it_adv(lx);
      }
      tmem_ld_wait();
      // re-bias the partial in TMEM while this step's math runs
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) tmem_st_32x32b_x8(tmem_base + b * BN + half * 64 + c8 * 8 + lane_off, kG128Magic);
      const float4* w4 = reinterpret_cast<const float4*>(ws_cur);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 w = w4[i];
        float2 s0 = make_float2(w.x, w.y), s1 = make_float2(w.z, w.w);
        if constexpr (MODE == G128_W4A4) {
          const float2 x2 = make_float2(xs_g, xs_g);
          s0 = f2_mul(x2, s0);  // dt32(xs * ws) / 16
          s1 = f2_mul(x2, s1);
        }
        const float2 p0 = f2_add(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])), neg_magic);
        const float2 p1 = f2_add(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])), neg_magic);
        acc[2 * i] = f2_fma(p0, s0, acc[2 * i]);
        acc[2 * i + 1] = f2_fma(p1, s1, acc[2 * i + 1]);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();  // also orders this step's ws_cur reads / ws_nxt writes
      if (lane == 0) mbar_arrive(&pempty[b]);
      if (++b == G128_NBUF) { b = 0; pph ^= 1; }

      if (cur.g == G - 1) {
        // tile done: scale, bias, round, store this thread's 64 columns
        const int row = cur.mb * Cfg::BM + quarter * 32 + lane;
        const int col0 = cur.nb * BN + half * 64;
        if (row < p.M && col0 < p.N) {
          const bool vec_ok = ((p.ldo % 8) == 0) && ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0);
          auto* orow = reinterpret_cast<typename EO::T*>(p.out) + (int64_t)row * p.ldo;
          const auto* bias = reinterpret_cast<const typename EO::T*>(p.bias);
#pragma unroll
          for (int c8 = 0; c8 < 8; ++c8) {
            const int c0 = col0 + c8 * 8;
            if (c0 < p.N) {
              const int n = min(8, p.N - c0);
              float y[8];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float a0 = acc[c8 * 4 + j].x, a1 = acc[c8 * 4 + j].y;
                if constexpr (MODE == G128_W4A8) {
                  a0 = __fmul_rn(a0, xs_row);  // dt32(acc * xs)
                  a1 = __fmul_rn(a1, xs_row);
                }
                y[2 * j] = a0;
                y[2 * j + 1] = a1;
              }
              if (bias != nullptr) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  if (j < n) y[j] = __fadd_rn(y[j], EO::to_f(bias[c0 + j]));
              }
#pragma unroll
              for (int j = 0; j < 8; ++j) y[j] = EO::round(y[j]);
              store8<OUT_DT>(orow + c0, y, vec_ok, n);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = make_float2(0.0f, 0.0f);
        if constexpr (MODE == G128_W4A8) {
          xs_row = xs_next;
          xs_next = load_xs(it_at(cur.tile + 2 * (int)gridDim.x));
        }
      }
      it_adv(cur);
      return true;
    };
    while (step_fn(std::integral_constant<int, 0>{}) && step_fn(std::integral_constant<int, 1>{}) &&
           step_fn(std::integral_constant<int, 2>{}) && step_fn(std::integral_constant<int, 3>{})) {
    }
  } else {
    regs_dec<64>();
    // ---------------- int4 -> 16*int4 unpack (warps 12..15) ----------------
    const int ctid = threadIdx.x - 32 * 12;
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      bool ok = true;
      for (int g = 0; g < G; ++g) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
        unpack_int4_slab_x16<BN, 128>(sBP + stage * Cfg::BP_BYTES, sB + stage * Cfg::B_BYTES, ctid);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// CTA-pair form (cta_group::2): 256x128 tiles, one 128-deep K slab = one scale
// group.  Each CTA TMA-loads its 128 rows of A and its 64 packed weight rows
// (its half of the tile's columns) onto its own `full` barrier; its unpack
// warpgroup expands the weight half to 16*q bytes and arrives on the
// leader's `conv` barrier (remotely from the peer); the leader's MMA warp
// issues M=256, N=128 MMAs whose A and B halves sit in the two CTAs' shared
// memory, accumulating each group's partial onto the 1.5*2^23 bias in one of
// four 128-column TMEM buffers, and commits `empty` / `pfull` to both CTAs.
// Each CTA's 8 epilogue warps fold the partials of their 32 rows x 64 columns
// into a 64-float register accumulator in group order (the single-CTA
// kernel's sequence) and leave through TMA stores; they release a partial
// buffer on a local barrier, and one thread per CTA forwards each release
// to the leader (a cluster-scope release from a warp with prefetch loads in
// flight would wait for them every group).  A CTA moves 56 KB through
// shared memory per 2.1 M MACs (its share of the pair's MMA) instead of the
// single-CTA tile's 80 KB.  16-bit outputs only.
struct G128PairCfg {
  static constexpr int BM = 128, BN = 128, BNH = 64, BK = 128;
  static constexpr int STAGES = 6;
  static constexpr int NBUF = 4;                   // TMEM partial buffers of BN columns
  static constexpr int BAR_BYTES = 320;            // barrier block + TMEM slot + abort flag
  static constexpr int CPW = BN / 2;               // columns per epilogue warp
  static constexpr int A_BYTES = BM * BK;          // 16 KB
  static constexpr int B_BYTES = BNH * BK;         // 16 KB unpacked
  static constexpr int BP_BYTES = BNH * BK / 2;    // 8 KB packed
  static constexpr int NUM_THREADS = 512;
  static constexpr int OUT_STAGE_BYTES = EPI_WARPS * EPI_STAGE_BYTES;
  static constexpr int WS_FLOATS = EPI_WARPS * 2 * CPW;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * (A_BYTES + B_BYTES + BP_BYTES) + OUT_STAGE_BYTES + BAR_BYTES + WS_FLOATS * 4 + 16;
  static_assert(3 * STAGES * 8 + 3 * NBUF * 8 + 16 + 16 <= BAR_BYTES, "barrier block overflows its reserve");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = NBUF * BN;
};

// tcgen05.wait::ld tied to the 16 registers of one tmem_ld_32x32b_x16.
__device__ __forceinline__ void tmem_ld_wait_regs16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

template <int MODE, int OUT_DT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(G128PairCfg::NUM_THREADS, 1)
    gemm_g128_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, G128Params p) {
  static_assert(OUT_DT == DT_BF16 || OUT_DT == DT_F16, "TMA-store epilogue: 16-bit outputs");
  using Cfg = G128PairCfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* sBP = sB + STAGES * Cfg::B_BYTES;
  uint8_t* sC = sBP + STAGES * Cfg::BP_BYTES;  // [EPI_WARPS][EPI_STAGE_BYTES] output staging
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + Cfg::OUT_STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;           // leader: both CTAs' weight halves unpacked (8 warps)
  constexpr int NBUF = Cfg::NBUF;
  constexpr int CPW = Cfg::CPW;
  uint64_t* pfull = conv + STAGES;           // [NBUF] partial of a group ready (both CTAs)
  uint64_t* pempty = pfull + NBUF;           // [NBUF] leader: both CTAs' partials consumed (2 forwards)
  uint64_t* lempty = pempty + NBUF;          // [NBUF] this CTA's 8 epilogue warps consumed the partial
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(lempty + NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 8);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&pempty[b], 2);
      mbar_init(&lempty[b], EPI_WARPS);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (p.M + 2 * Cfg::BM - 1) / (2 * Cfg::BM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int G = p.K / Cfg::BK;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp < 4) {
    regs_dec<64>();
    if (warp == 0 && lane == 0) {
      // ---------------- TMA producer (both CTAs: own halves, own barrier) ----------------
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        const int arow = mb * 2 * Cfg::BM + (int)rank * Cfg::BM;
        const int brow = nb * BN + (int)rank * Cfg::BNH;
        for (int g = 0; g < G; ++g) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::BP_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], g * Cfg::BK, arow);
          tma_load_2d(sBP + stage * Cfg::BP_BYTES, &tmB, &full[stage], g * (Cfg::BK / 2), brow);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    } else if (warp == 1 && leader && lane == 0) {
      // ---------------- MMA issuer (leader CTA only) ----------------
      constexpr uint32_t idesc = umma_idesc_i8(2 * Cfg::BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int b = 0;
      uint32_t pph = 0;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        for (int g = 0; g < G; ++g) {
          if (!mbar_wait_bounded(&conv[stage], phase, abort_flag) ||
              !mbar_wait_bounded(&pempty[b], pph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_k_sw128(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bdesc = umma_desc_k_sw128(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < Cfg::BK / 32; ++k)  // accumulate onto the 1.5*2^23 bias
            umma_i8_pair(tmem_base + b * BN, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
          umma_commit_pair(&empty[stage], 0x3);
          umma_commit_pair(&pfull[b], 0x3);
          if (++b == NBUF) { b = 0; pph ^= 1; }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    } else if (warp == 2 && lane == 0) {
      // ---------------- release forwarder (both CTAs) ----------------
      // One remote arrival on the leader's pempty[b] per completion of this
      // CTA's local lempty[b] (8 epilogue warps): the NBUF initial releases,
      // then one per (tile, group).  The epilogue warps arrive locally, so
      // their cluster-scope release never waits on their prefetch loads.
      const uint32_t pempty_leader = mapa_shared(smem_u32(&pempty[0]), 0);  // + 8*b
      int tiles = 0;
      for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) ++tiles;
      const int64_t releases = (int64_t)NBUF + (int64_t)tiles * G;
      int b = 0;
      uint32_t ph = 0;
      for (int64_t i = 0; i < releases; ++i) {
        if (!mbar_wait_bounded(&lempty[b], ph, abort_flag)) break;
        mbar_arrive_cluster(pempty_leader + 8u * b);
        if (++b == NBUF) { b = 0; ph ^= 1; }
      }
    }
  } else if (warp < 12) {
    regs_inc<192>();
    // ---------------- epilogue (both CTAs) ----------------
    const int quarter = warp & 3;        // TMEM lanes 32*quarter.. (warp % 4 rule)
    const int half = (warp - 4) >> 2;    // tile columns CPW*half..
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
#pragma unroll 1
    for (int b = 0; b < NBUF; ++b)
#pragma unroll
      for (int c8 = 0; c8 < CPW / 8; ++c8)
        tmem_st_32x32b_x8(tmem_base + b * BN + half * CPW + c8 * 8 + lane_off, kG128Magic);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < NBUF; ++b) mbar_arrive(&lempty[b]);

    // A step is one (tile, group) in issue order.  Each warp stages the CPW
    // column scales of its half of the tile in its own shared-memory buffer
    // (double-buffered by step parity); every lane loads two of them, five
    // steps ahead, into a 4-slot register ring (static slots: the step loop
    // is unrolled by 4).  W4A4 row scales travel four steps ahead the same way.
    struct It {
      int tile, g, mb, nb;
    };
    auto it_at = [&](int tile) {
      It t{tile, 0, 0, 0};
      if (tile < num_tiles) tile_coords(tile, num_m, num_n, t.mb, t.nb);
      return t;
    };
    auto it_adv = [&](It& t) {
      if (++t.g == G) {
        t.g = 0;
        t.tile += num_clusters;
        if (t.tile < num_tiles) tile_coords(t.tile, num_m, num_n, t.mb, t.nb);
      }
    };
    auto load_ws = [&](const It& t, int j) -> float {  // column CPW*half + 32*j + lane
      if (t.tile >= num_tiles) return 0.0f;
      return g128_wscale16(p, G, t.nb * BN + half * CPW + 32 * j + lane, t.g);
    };
    auto row_of = [&](const It& t) { return t.mb * 2 * Cfg::BM + (int)rank * Cfg::BM + quarter * 32 + lane; };
    auto load_xs = [&](const It& t) -> float {
      if (t.tile >= num_tiles) return 0.0f;
      const int row2 = row_of(t);
      if (row2 >= p.M) return 0.0f;
      if constexpr (MODE == G128_W4A8) return __ldg(p.a_scale + row2);
      else return __ldg(p.a_scale + (int64_t)row2 * G + t.g);
    };

    float* wbuf = s_ws + (warp - 4) * 2 * CPW;  // [2][CPW] floats of this warp
    uint8_t* stage_out = sC + (warp - 4) * EPI_STAGE_BYTES;
    It cur = it_at(cluster_id);
    It la = cur;
    constexpr int JW = CPW / 32;  // scales per lane
#pragma unroll
    for (int j = 0; j < JW; ++j) wbuf[32 * j + lane] = load_ws(la, j);
    float rw[4][JW];  // scales of step t in slot t % 4 (steps 1..4 ahead)
#pragma unroll
    for (int k = 1; k <= 4; ++k) {
      it_adv(la);
#pragma unroll
      for (int j = 0; j < JW; ++j) rw[k & 3][j] = load_ws(la, j);
    }
    it_adv(la);  // step 5
    It lx = cur;
    float rxs[4];
    if constexpr (MODE == G128_W4A4) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        rxs[k] = load_xs(lx);
        it_adv(lx);
      }
    }
    float xs_row = 0.0f, xs_next = 0.0f;
    if constexpr (MODE == G128_W4A8) {
      xs_row = load_xs(cur);
      xs_next = load_xs(it_at(cur.tile + num_clusters));
    }
    __syncwarp();

    float2 acc[CPW / 2];
#pragma unroll
    for (int j = 0; j < CPW / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    int b = 0;
    uint32_t pph = 0;

    auto step_fn = [&](auto kc) -> bool {
      constexpr int K = decltype(kc)::value;
      constexpr int K1 = (K + 1) & 3;
      if (cur.tile >= num_tiles) return false;
      const bool ok = mbar_wait_bounded(&pfull[b], pph, abort_flag);
      if (__any_sync(0xffffffffu, !ok || *abort_flag)) return false;
      tc_fence_after();
      const uint32_t tb = tmem_base + b * BN + half * CPW + lane_off;
      static_assert(CPW == 64, "two 32-column TMEM loads per step");
      uint32_t r[64];
      tmem_ld_32x32b_x32(tb, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_ld_32x32b_x32(tb + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      const float* ws_cur = wbuf + (K & 1) * CPW;
      float* ws_nxt = wbuf + (K1 & 1) * CPW;
#pragma unroll
      for (int j = 0; j < JW; ++j) {
        ws_nxt[32 * j + lane] = rw[K1][j];
        rw[K1][j] = load_ws(la, j);  // step + 5
      }
      it_adv(la);
      float xs_g = 0.0f;
      if constexpr (MODE == G128_W4A4) {
        xs_g = rxs[K];
        rxs[K] = load_xs(lx);
        it_adv(lx);
      }
      tmem_ld_wait();
      // re-bias the partial in TMEM while this step's math runs
#pragma unroll
      for (int c8 = 0; c8 < CPW / 8; ++c8) tmem_st_32x32b_x8(tb + c8 * 8, kG128Magic);
      const float4* w4 = reinterpret_cast<const float4*>(ws_cur);
#pragma unroll
      for (int i = 0; i < CPW / 4; ++i) {
        const float4 w = w4[i];
        float2 s0 = make_float2(w.x, w.y), s1 = make_float2(w.z, w.w);
        if constexpr (MODE == G128_W4A4) {
          const float2 x2 = make_float2(xs_g, xs_g);
          s0 = f2_mul(x2, s0);  // dt32(xs * ws) / 16
          s1 = f2_mul(x2, s1);
        }
        const float2 p0 = f2_add(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])), neg_magic);
        const float2 p1 = f2_add(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])), neg_magic);
        acc[2 * i] = f2_fma(p0, s0, acc[2 * i]);
        acc[2 * i + 1] = f2_fma(p1, s1, acc[2 * i + 1]);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();  // also orders this step's ws_cur reads / ws_nxt writes
      if (lane == 0) mbar_arrive(&lempty[b]);
      if (++b == NBUF) { b = 0; pph ^= 1; }

      if (cur.g == G - 1) {
        // tile done: row scale (W4A8), bias, one rounding, TMA stores
        const int row_base = cur.mb * 2 * Cfg::BM + (int)rank * Cfg::BM + quarter * 32;
        const int colh = cur.nb * BN + half * CPW;
        const uint16_t* bias = reinterpret_cast<const uint16_t*>(p.bias);
#pragma unroll
        for (int c4 = 0; c4 < CPW / 32; ++c4) {  // static acc indices
          const int col0 = colh + c4 * 32;
          if (row_base >= p.M || col0 >= p.N) continue;  // warp-uniform
          // the chunk's 32 bias values, the same for every lane (broadcast loads)
          uint32_t bw[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) bw[j] = 0u;
          if (bias != nullptr) {
            if (col0 + 32 <= p.N) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(bias + col0) + q);
                bw[4 * q] = v.x; bw[4 * q + 1] = v.y; bw[4 * q + 2] = v.z; bw[4 * q + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const uint32_t lo = col0 + 2 * j < p.N ? (uint32_t)__ldg(bias + col0 + 2 * j) : 0u;
                const uint32_t hi = col0 + 2 * j + 1 < p.N ? (uint32_t)__ldg(bias + col0 + 2 * j + 1) : 0u;
                bw[j] = lo | (hi << 16);
              }
            }
          }
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float a0 = acc[c4 * 16 + j].x, a1 = acc[c4 * 16 + j].y;
            if constexpr (MODE == G128_W4A8) {
              a0 = __fmul_rn(a0, xs_row);  // dt32(acc * xs)
              a1 = __fmul_rn(a1, xs_row);
            }
            if (bias != nullptr) {
              if constexpr (OUT_DT == DT_BF16) {
                a0 = __fadd_rn(a0, __uint_as_float(bw[j] << 16));
                a1 = __fadd_rn(a1, __uint_as_float(bw[j] & 0xFFFF0000u));
              } else {
                const float2 bf = __half22float2(*reinterpret_cast<const __half2*>(&bw[j]));
                a0 = __fadd_rn(a0, bf.x);
                a1 = __fadd_rn(a1, bf.y);
              }
            }
            if constexpr (OUT_DT == DT_BF16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(a0, a1);
              w[j] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(a0, a1);
              w[j] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<uint4*>(stage_out + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stage_out, col0, row_base);
            bulk_commit_group();
          }
        }
#pragma unroll
        for (int j = 0; j < CPW / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
        if constexpr (MODE == G128_W4A8) {
          xs_row = xs_next;
          xs_next = load_xs(it_at(cur.tile + 2 * num_clusters));
        }
      }
      it_adv(cur);
      return true;
    };
    while (step_fn(std::integral_constant<int, 0>{}) && step_fn(std::integral_constant<int, 1>{}) &&
           step_fn(std::integral_constant<int, 2>{}) && step_fn(std::integral_constant<int, 3>{})) {
    }
    if (lane == 0) bulk_wait_all();  // TMA stores complete before exit
  } else {
    regs_dec<64>();
    // ---------------- int4 -> 16*int4 unpack of this CTA's weight half ----------------
    const int ctid = threadIdx.x - 32 * 12;
    const uint32_t conv_leader0 = mapa_shared(smem_u32(&conv[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      bool ok = true;
      for (int g = 0; g < G; ++g) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
        unpack_int4_slab_x16<Cfg::BNH, 128>(sBP + stage * Cfg::BP_BYTES, sB + stage * Cfg::B_BYTES, ctid);
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(conv_leader0 + stage * (uint32_t)sizeof(uint64_t));
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
    }
  }

  tc_fence_before();
  cluster_sync();  // all MMAs done and all remote arrivals delivered
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace qlin
