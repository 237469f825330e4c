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
// CTA-pair form (cta_group::2): 256x128 tiles; one pipeline step covers two
// scale groups (a 256-deep K slab), so the per-step handshakes (ring
// barriers, MMA commits, partial-buffer releases) are paid once per two
// groups.  12 warps per CTA:
//   warp 0      TMA producer: this CTA's 128 activation rows (two 128-byte
//               swizzled boxes) and its 64 packed weight rows of the step
//               onto its own `full` barrier
//   warp 1      TMEM allocator; on the leader the MMA issuer (M=256, N=128,
//               K=32 x 8 per step, each group's partial accumulated onto the
//               1.5*2^23 bias in its own 128-column half of a 256-column
//               TMEM buffer, two buffers), on the peer the release forwarder
//   warps 2-3   nibble unpack of this CTA's weight half to 16*q bytes, one
//               group each
//   warps 4-11  epilogue: two warps per TMEM lane quarter, 64 columns each;
//               per step the two groups' partials are folded into a 64-float
//               register accumulator in group order (the single-CTA kernel's
//               sequence); TMA stores at the tile's end
// Partial-buffer release: the leader's epilogue warps arrive on the leader's
// `pempty` directly; the peer's arrive on its local `lempty`, and the peer's
// warp 1 forwards each completion with one remote arrival to the leader's
// `pempty`.  Remote arrivals carry release semantics at CTA scope, as
// CUTLASS's cluster barriers do: a cluster-scope release made every arrival
// wait for the memory system (about 1200 cycles each, measured).
// K must be a multiple of 256; 16-bit outputs only.
struct G128PairCfg {
  static constexpr int BM = 128, BN = 128, BNH = 64, BK = 128;
  static constexpr int GPS = 2;                    // scale groups per pipeline step
  static constexpr int KS = GPS * BK;              // K depth of a step
  static constexpr int STAGES = 3;
  static constexpr int NBUF = 2;                   // TMEM buffers of GPS * BN columns
  static constexpr int EPI_W = 8;                  // epilogue warps
  static constexpr int EPI_WARP0 = 4;              // first epilogue warp
  static constexpr int CPW = BN / 2;               // columns per epilogue warp
  static constexpr int BAR_BYTES = 256;            // barrier block + TMEM slot + abort flag
  static constexpr int A_BYTES = BM * KS;          // 32 KB (two 128-byte boxes)
  static constexpr int B_BYTES = BNH * KS;         // 16 KB unpacked (two [64][128] slabs)
  static constexpr int BP_BYTES = BNH * KS / 2;    // 8 KB packed
  static constexpr int NUM_THREADS = 32 * (EPI_WARP0 + EPI_W);
  static constexpr int OUT_STAGE_BYTES = EPI_W * EPI_STAGE_BYTES;
  static constexpr int WS_FLOATS = EPI_W * 2 * GPS * CPW;  // [warp][step parity][group][column]
  static constexpr int SMEM_BYTES =
      1024 + STAGES * (A_BYTES + B_BYTES + BP_BYTES) + OUT_STAGE_BYTES + BAR_BYTES + WS_FLOATS * 4 + 16;
  static_assert(3 * STAGES * 8 + 3 * NBUF * 8 + 8 + 16 <= BAR_BYTES, "barrier block overflows its reserve");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static constexpr uint32_t TMEM_COLS = NBUF * GPS * BN;
};


// Nibble unpack of a [64 rows][KS/2 packed bytes] slab's 64-byte group
// column `grp` into the 128-byte swizzled [64][128] int8 layout (16*q per
// byte) by one warp.
__device__ __forceinline__ void unpack_int4_group64_warp(const uint8_t* src, uint8_t* dst, int grp, int lane) {
  constexpr int SRC_ROW = G128PairCfg::KS / 2;  // packed bytes per row of the step
  const int c = lane & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint2 pk[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = (lane >> 3) + 4 * (8 * h + k);
      pk[k] = *reinterpret_cast<const uint2*>(src + row * SRC_ROW + grp * 64 + c * 8);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = (lane >> 3) + 4 * (8 * h + k);
      const uint32_t l0 = (pk[k].x << 4) & 0xF0F0F0F0u, h0 = pk[k].x & 0xF0F0F0F0u;
      const uint32_t l1 = (pk[k].y << 4) & 0xF0F0F0F0u, h1 = pk[k].y & 0xF0F0F0F0u;
      *reinterpret_cast<uint4*>(dst + row * 128 + ((c ^ (row & 7)) << 4)) =
          make_uint4(__byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362), __byte_perm(l1, h1, 0x5140),
                     __byte_perm(l1, h1, 0x7362));
    }
  }
}

template <int MODE, int OUT_DT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(G128PairCfg::NUM_THREADS, 1)
    gemm_g128_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, G128Params p) {
  static_assert(OUT_DT == DT_BF16 || OUT_DT == DT_F16, "TMA-store epilogue: 16-bit outputs");
  using Cfg = G128PairCfg;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  constexpr int NBUF = Cfg::NBUF;
  constexpr int CPW = Cfg::CPW;
  constexpr int GPS = Cfg::GPS;
  constexpr int BUFW = GPS * BN;  // TMEM columns of one buffer
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;                          // [STAGES][GPS][128 rows][128 B]
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;    // [STAGES][GPS][64 rows][128 B]
  uint8_t* sBP = sB + STAGES * Cfg::B_BYTES;   // [STAGES][64 rows][KS/2 B]
  uint8_t* sC = sBP + STAGES * Cfg::BP_BYTES;  // [EPI_W][EPI_STAGE_BYTES] output staging
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + Cfg::OUT_STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;    // leader: both CTAs' weight halves unpacked (4 arrivals)
  uint64_t* pfull = conv + STAGES;    // [NBUF] partials of a step ready (both CTAs)
  uint64_t* lempty = pfull + NBUF;    // [NBUF] peer: its 8 epilogue warps consumed the partials
  uint64_t* pempty = lempty + NBUF;   // [NBUF] leader: 8 local epilogue warps + the peer's forward
  uint64_t* drain = pempty + NBUF;    // abort path: the MMA issuer's last commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
      mbar_init(&conv[s], 2 * GPS);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&pfull[b], 1);
      mbar_init(&lempty[b], Cfg::EPI_W);
      mbar_init(&pempty[b], Cfg::EPI_W + 1);
    }
    mbar_init(drain, 1);
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
  const int G = p.K / Cfg::BK;   // scale groups (even)
  const int S = G / GPS;         // steps per tile
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs: own halves, own barrier) ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      ArmedLoads armed;
      bool ok = true;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        const int arow = mb * 2 * Cfg::BM + (int)rank * Cfg::BM;
        const int brow = nb * BN + (int)rank * Cfg::BNH;
        for (int st = 0; st < S; ++st) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::BP_BYTES);
#pragma unroll
          for (int j = 0; j < GPS; ++j)
            tma_load_2d(sA + stage * Cfg::A_BYTES + j * (Cfg::BM * Cfg::BK), &tmA, &full[stage],
                        (st * GPS + j) * Cfg::BK, arow);
          tma_load_2d(sBP + stage * Cfg::BP_BYTES, &tmB, &full[stage], st * (Cfg::KS / 2), brow);
          armed.note(stage, phase);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) armed.drain(full, STAGES);  // no load still writing shared memory at exit
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------- MMA issuer (leader CTA only) ----------------
      constexpr uint32_t idesc = umma_idesc_i8(2 * Cfg::BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int b = 0;
      uint32_t pph = 0;
      bool ok = true, issued = false;
      for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
        for (int st = 0; st < S; ++st) {
          if (!mbar_wait_bounded(&conv[stage], phase, abort_flag) || !mbar_wait_bounded(&pempty[b], pph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < GPS; ++j) {
            const uint64_t adesc = umma_desc_k_sw128(smem_u32(sA + stage * Cfg::A_BYTES + j * (Cfg::BM * Cfg::BK)));
            const uint64_t bdesc = umma_desc_k_sw128(smem_u32(sB + stage * Cfg::B_BYTES + j * (Cfg::BNH * Cfg::BK)));
#pragma unroll
            for (int k = 0; k < Cfg::BK / 32; ++k)  // accumulate onto the 1.5*2^23 bias
              umma_i8_pair(tmem_base + b * BUFW + j * BN, adesc + 2 * k, bdesc + 2 * k, idesc, 1u);
          }
          issued = true;
          umma_commit_pair(&empty[stage], 0x3);
          umma_commit_pair(&pfull[b], 0x3);
          if (++b == NBUF) { b = 0; pph ^= 1; }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag && issued) {  // MMAs complete before TMEM is released
        umma_commit_pair(drain, 0x1);
        mbar_wait_drain(drain, 0);
      }
    } else if (!leader && lane == 0) {
      // ---------------- release forwarder (peer CTA) ----------------
      // one remote arrival on the leader's pempty[b] per completion of this
      // CTA's lempty[b]: the NBUF initial releases, then one per (tile, step)
      const uint32_t pempty_leader = mapa_shared(smem_u32(&pempty[0]), 0);  // + 8*b
      int tiles = 0;
      for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) ++tiles;
      const int64_t releases = (int64_t)NBUF + (int64_t)tiles * S;
      int b = 0;
      uint32_t ph = 0;
      for (int64_t i = 0; i < releases; ++i) {
        if (!mbar_wait_bounded(&lempty[b], ph, abort_flag)) break;
        mbar_arrive_remote(pempty_leader + 8u * b);
        if (++b == NBUF) { b = 0; ph ^= 1; }
      }
    }
  } else if (warp < Cfg::EPI_WARP0) {
    // ---------------- int4 -> 16*int4 unpack (warp 2 + j: group j of every step) ----------------
    const int grp = warp - 2;
    const uint32_t conv_leader0 = mapa_shared(smem_u32(&conv[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = cluster_id; ok && tile < num_tiles; tile += num_clusters) {
      for (int st = 0; st < S; ++st) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
        unpack_int4_group64_warp(sBP + stage * Cfg::BP_BYTES, sB + stage * Cfg::B_BYTES + grp * (Cfg::BNH * Cfg::BK),
                                 grp, lane);
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&conv[stage]);
          else mbar_arrive_remote(conv_leader0 + stage * (uint32_t)sizeof(uint64_t));
        }
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ---------------- epilogue (both CTAs, 8 warps) ----------------
    const int ew = warp - Cfg::EPI_WARP0;  // 0..7
    const int quarter = warp & 3;          // TMEM lanes 32*quarter.. (warp % 4 rule)
    const int half = ew >> 2;              // tile columns CPW*half..
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint64_t* release = leader ? pempty : lempty;
#pragma unroll 1
    for (int c = 0; c < NBUF * GPS; ++c)
#pragma unroll
      for (int c8 = 0; c8 < CPW / 8; ++c8)
        tmem_st_32x32b_x8(tmem_base + c * BN + half * CPW + c8 * 8 + lane_off, kG128Magic);
    tmem_st_wait();
    tc_fence_before();
    __syncwarp();
    if (lane == 0)
      for (int b = 0; b < NBUF; ++b) mbar_arrive(&release[b]);

    // A step is one (tile, pair of groups) in issue order.  During step t
    // each lane loads the scales of its two columns (lane, lane + 32) in both
    // groups of step t + 1 (the tile's scale rows stay in L1) and stages them
    // at the end of the step in the warp's shared-memory buffer
    // (double-buffered by step parity); the fold reads them back as broadcast
    // float4 loads.  W4A4 row scales are loaded one step ahead into
    // registers.  The next tile's coordinates are computed once per tile.
    int tile = cluster_id, st = 0, mb = 0, nb = 0, nmb = 0, nnb = 0;
    if (tile < num_tiles) tile_coords(tile, num_m, num_n, mb, nb);
    if (tile + num_clusters < num_tiles) tile_coords(tile + num_clusters, num_m, num_n, nmb, nnb);
    const int lcol = half * CPW + lane;                          // first column of this lane in a tile
    const int lrow = (int)rank * Cfg::BM + quarter * 32 + lane;  // this lane's row within a tile
    float* wbuf = s_ws + ew * 2 * GPS * CPW;  // [step parity][group][CPW] floats of this warp
    uint8_t* stage_out = sC + ew * EPI_STAGE_BYTES;
    // scales (and W4A4 row scales) of the step after (tile, st)
    auto next_pos = [&](int& t2, int& n2, int& m2, int& g2) {
      const bool same = st + 1 < S;
      t2 = same ? tile : tile + num_clusters;
      n2 = same ? nb : nnb;
      m2 = same ? mb : nmb;
      g2 = same ? (st + 1) * GPS : 0;
    };
    auto load_ws = [&](float (&w)[2 * GPS], int t2, int n2, int g2) {
#pragma unroll
      for (int j = 0; j < GPS; ++j) {
        w[2 * j] = t2 < num_tiles ? g128_wscale16(p, G, n2 * BN + lcol, g2 + j) : 0.0f;
        w[2 * j + 1] = t2 < num_tiles ? g128_wscale16(p, G, n2 * BN + lcol + 32, g2 + j) : 0.0f;
      }
    };
    auto stage_ws = [&](int par, const float (&w)[2 * GPS]) {
      float* dst = wbuf + par * GPS * CPW;
#pragma unroll
      for (int j = 0; j < GPS; ++j) {
        dst[j * CPW + lane] = w[2 * j];
        dst[j * CPW + 32 + lane] = w[2 * j + 1];
      }
    };
    {
      float w0[2 * GPS];
      load_ws(w0, tile, nb, 0);
      stage_ws(0, w0);
    }
    float xg[GPS] = {};  // W4A4: row scales of the current step's groups
    float xs_row = 0.0f;  // W4A8: row scale of the current tile
    if (tile < num_tiles && mb * 2 * Cfg::BM + lrow < p.M) {
      const int64_t row = mb * 2 * Cfg::BM + lrow;
      if constexpr (MODE == G128_W4A8) {
        xs_row = __ldg(p.a_scale + row);
      } else {
#pragma unroll
        for (int j = 0; j < GPS; ++j) xg[j] = __ldg(p.a_scale + row * G + j);
      }
    }
    __syncwarp();

    float2 acc[CPW / 2];
#pragma unroll
    for (int j = 0; j < CPW / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
    const float2 neg_magic = make_float2(-12582912.0f, -12582912.0f);
    int b = 0;
    uint32_t pph = 0;
    int par = 0;

    // fold one 32-column chunk (columns 32*h.. of this warp, group j of the
    // step) from its TMEM registers
    auto fold = [&](const uint32_t (&r)[32], auto jc, auto hc, const float* ws_step) {
      constexpr int j = decltype(jc)::value, h = decltype(hc)::value;
      const float4* w4 = reinterpret_cast<const float4*>(ws_step + j * CPW + 32 * h);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 w = w4[i];
        float2 s0 = make_float2(w.x, w.y), s1 = make_float2(w.z, w.w);
        if constexpr (MODE == G128_W4A4) {
          const float2 x2 = make_float2(xg[j], xg[j]);
          s0 = f2_mul(x2, s0);  // dt32(xs * ws) / 16
          s1 = f2_mul(x2, s1);
        }
        const float2 p0 = f2_add(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])), neg_magic);
        const float2 p1 = f2_add(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])), neg_magic);
        acc[16 * h + 2 * i] = f2_fma(p0, s0, acc[16 * h + 2 * i]);
        acc[16 * h + 2 * i + 1] = f2_fma(p1, s1, acc[16 * h + 2 * i + 1]);
      }
    };

#pragma unroll 1
    while (tile < num_tiles) {
      const bool ok = mbar_wait_bounded(&pfull[b], pph, abort_flag);
      if (__any_sync(0xffffffffu, !ok || *abort_flag)) break;
      tc_fence_after();
      // chunk c = (group c >> 1, column half c & 1): TMEM column b*BUFW + (c>>1)*BN + half*CPW + 32*(c&1)
      const uint32_t tb = tmem_base + b * BUFW + half * CPW + lane_off;
      const float* ws_step = wbuf + par * GPS * CPW;
      uint32_t ra[32], rb[32];
      tmem_ld_32x32b_x32(tb, ra);
      int t2, n2, m2, g2;
      next_pos(t2, n2, m2, g2);
      float wn[2 * GPS];  // staged at the end of this step
      load_ws(wn, t2, n2, g2);
      float xn[GPS] = {};
      if constexpr (MODE == G128_W4A4) {
        const int64_t row2 = (int64_t)m2 * 2 * Cfg::BM + lrow;
        if (t2 < num_tiles && row2 < p.M) {
#pragma unroll
          for (int j = 0; j < GPS; ++j) xn[j] = __ldg(p.a_scale + row2 * G + g2 + j);
        }
      }
      // four 32-column chunks (group, column half), the next one in flight
      // while the current one is folded
      tmem_ld_wait_regs(ra);
      tmem_ld_32x32b_x32(tb + 32, rb);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) tmem_st_32x32b_x8(tb + c8 * 8, kG128Magic);
      fold(ra, std::integral_constant<int, 0>{}, std::integral_constant<int, 0>{}, ws_step);
      tmem_ld_wait_regs(rb);
      tmem_ld_32x32b_x32(tb + BN, ra);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) tmem_st_32x32b_x8(tb + 32 + c8 * 8, kG128Magic);
      fold(rb, std::integral_constant<int, 0>{}, std::integral_constant<int, 1>{}, ws_step);
      tmem_ld_wait_regs(ra);
      tmem_ld_32x32b_x32(tb + BN + 32, rb);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) tmem_st_32x32b_x8(tb + BN + c8 * 8, kG128Magic);
      fold(ra, std::integral_constant<int, 1>{}, std::integral_constant<int, 0>{}, ws_step);
      tmem_ld_wait_regs(rb);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) tmem_st_32x32b_x8(tb + BN + 32 + c8 * 8, kG128Magic);
      fold(rb, std::integral_constant<int, 1>{}, std::integral_constant<int, 1>{}, ws_step);
      stage_ws(par ^ 1, wn);  // the other buffer: last read by the previous step
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();  // orders this step's ws_step reads and the staged scales
      if (lane == 0) mbar_arrive(&release[b]);
      if (++b == NBUF) { b = 0; pph ^= 1; }
      par ^= 1;
      if constexpr (MODE == G128_W4A4) {
#pragma unroll
        for (int j = 0; j < GPS; ++j) xg[j] = xn[j];
      }

      if (st == S - 1) {
        // tile done: row scale (W4A8), bias, one rounding, TMA stores of
        // two 32x32 chunks, eight columns at a time into the swizzled staging
        const int row_base = mb * 2 * Cfg::BM + (int)rank * Cfg::BM + quarter * 32;
        const uint16_t* bias = reinterpret_cast<const uint16_t*>(p.bias);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col0 = nb * BN + half * CPW + 32 * h;
          if (row_base >= p.M || col0 >= p.N) continue;  // warp-uniform
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // the chunk's 8 bias values, the same for every lane (broadcast loads)
            uint32_t bw[4] = {0u, 0u, 0u, 0u};
            const int c = col0 + 8 * k;
            if (bias != nullptr) {
              if (c + 8 <= p.N) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(bias + c));
                bw[0] = v.x; bw[1] = v.y; bw[2] = v.z; bw[3] = v.w;
              } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t lo = c + 2 * j < p.N ? (uint32_t)__ldg(bias + c + 2 * j) : 0u;
                  const uint32_t hi = c + 2 * j + 1 < p.N ? (uint32_t)__ldg(bias + c + 2 * j + 1) : 0u;
                  bw[j] = lo | (hi << 16);
                }
              }
            }
            uint32_t w[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float a0 = acc[16 * h + 4 * k + j].x, a1 = acc[16 * h + 4 * k + j].y;
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
                __nv_bfloat162 hh = __floats2bfloat162_rn(a0, a1);
                w[j] = *reinterpret_cast<uint32_t*>(&hh);
              } else {
                __half2 hh = __floats2half2_rn(a0, a1);
                w[j] = *reinterpret_cast<uint32_t*>(&hh);
              }
            }
            *reinterpret_cast<uint4*>(stage_out + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&tmC, stage_out, col0, row_base);
            bulk_commit_group();
          }
        }
#pragma unroll
        for (int j = 0; j < CPW / 2; ++j) acc[j] = make_float2(0.0f, 0.0f);
        // next tile: coordinates, the one after it, and (W4A8) its row scale,
        // needed at its end
        tile += num_clusters;
        mb = nmb;
        nb = nnb;
        if (tile + num_clusters < num_tiles) tile_coords(tile + num_clusters, num_m, num_n, nmb, nnb);
        if constexpr (MODE == G128_W4A8)
          xs_row = (tile < num_tiles && mb * 2 * Cfg::BM + lrow < p.M) ? __ldg(p.a_scale + mb * 2 * Cfg::BM + lrow)
                                                                        : 0.0f;
        st = 0;
      } else {
        ++st;
      }
    }
    if (lane == 0) bulk_wait_all();  // TMA stores complete before exit
  }

  tc_fence_before();
  cluster_sync();  // all MMAs done and all remote arrivals delivered
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace qlin
