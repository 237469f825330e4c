// Persistent warp-specialised int8 GEMM on the sm_100a 5th-generation tensor
// cores: C[M,N] = A[M,K] . B[N,K]^T, int32 accumulation in tensor memory.
//
//   warp 0      TMA producer: A and B K-slabs (128 bytes of K per stage,
//               128B-swizzled) into a STAGES-deep shared-memory ring;
//               for packed-int4 B it loads the packed slab instead.
//   warp 1      TMEM allocator + MMA issuer: tcgen05.mma.kind::i8 (M=128,
//               N=BN, K=32) x 4 per stage, commits free the ring slot and,
//               at tile end, hand the accumulator to the epilogue.
//   warps 2-9   epilogue: tcgen05.ld of the int32 tile (two warps per
//               32-lane TMEM quarter, each converting half of the columns),
//               the reference's scale/bias/rounding sequence, stores to HBM.
//               Two TMEM accumulators let the epilogue of tile i overlap the
//               MMAs of tile i+1.
//   warps 10-13 (packed-int4 B only) nibble -> int8 unpack of the B slab
//               into the swizzled operand layout the MMA reads.
//
// No TMA multicast is used anywhere (the same kernel runs in multi-GPU jobs).
// Every pipeline wait is bounded: on timeout the kernel sets a device error
// word, all roles leave their loops, TMEM is released and the kernel exits.
#pragma once

#include "common.cuh"

namespace qlin {

// Device error word (bit 0: a pipeline wait timed out; bit 2: after a
// timeout, the kernel's in-flight TMA loads or MMAs did not drain within the
// limit either).  Read and cleared by qlin_device_error().  Defined here:
// gemm.cu is the only translation unit that includes this header.
__device__ uint32_t g_error_bits = 0;

// Pipeline waits give up after this many nanoseconds and flag the failure
// (qlin_set_wait_limit; 2 s by default).
__device__ uint64_t g_wait_limit_ns = 2000000000ull;

// Bounded wait on an mbarrier phase.  Returns false (and sets the device
// error word and *abort) if the phase did not complete within the limit or
// another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
  const uint64_t t0 = globaltimer_ns();
  uint32_t iter = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++iter & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit) {
        atomicOr(&g_error_bits, 1u);
        *abort = 1;
        return false;
      }
    }
  }
}

// Abort path: wait (bounded, whatever the abort flag says) for a phase that
// completes once asynchronous work this thread issued earlier has finished.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit) {
      atomicOr(&g_error_bits, 4u);
      return;
    }
  }
}

// TMA loads a producer thread armed on the `full` barriers of the operand
// ring: bit s of `armed` once stage s was filled, bit s of `par` the phase
// parity of its last fill.  Before the producer leaves its role it waits for
// those last fills, so no load is still writing shared memory when the CTA
// exits -- after an abort too, when the MMA issuer never consumed them.  (On
// the normal path the last fills land within microseconds, while the MMA
// issuer is still consuming them.)
struct ArmedLoads {
  uint32_t armed = 0, par = 0;
  __device__ __forceinline__ void note(int stage, uint32_t phase) {
    armed |= 1u << stage;
    par = (par & ~(1u << stage)) | (phase << stage);
  }
  __device__ __forceinline__ void drain(uint64_t* full, int stages) const {
    for (int s = 0; s < stages; ++s)
      if (armed >> s & 1u) mbar_wait_drain(&full[s], par >> s & 1u);
  }
};

enum : int {
  EPI_W8A8_ROW = 0,     // dt(dt(float(acc)*xs[m]*ws[n]) + bias[n])
  EPI_W8A8_TENSOR = 1,  // dt(dt(float(acc)*(ws*xs[m])) + bias[n])
  EPI_W4A4_ROW = 2,     // dt(float(acc)*xs[m]*ws[n] + float(bias[n]))
  EPI_I32 = 3,          // raw int32
  EPI_POST = 8,         // flag on the W8A8 epilogues: GELU / residual + gate after them
};
constexpr int epi_base(int epi) { return epi & 7; }

constexpr int kMaxOutputs = 8;  // destinations of one GEMM (tensor-parallel gather)

struct GemmParams {
  int M, N, K;
  const float* a_scale;  // [M]
  const float* w_scale;  // [N] or [1]
  const void* bias;      // [N] in the output dtype, or null
  void* out;             // [M, ldo] output (the only destination when nout == 1)
  int64_t ldo;           // output row stride (elements)
  int num_sms;
  int nout;              // number of destinations
  int64_t col_off;       // column of this GEMM's column 0 in every destination
  void* outs[kMaxOutputs];  // destinations when nout > 1 (peer buffers)
  // EPI_POST steps (16-bit outputs): y = dt(gelu_tanh(y)) for columns >=
  // gelu_col0, then y = dt(residual + dt(gate * y)) (dt(residual + y)
  // without a gate); residual [M, ld_res], gate row = row / rows_per_gate
  int64_t gelu_col0;
  const void* residual;
  int64_t ld_res;
  const void* gate;
  int64_t gate_ld;
  int64_t rows_per_gate;
  // Failure-detection self-test only (qlin_selftest_gemm_stall): the
  // producer leaves this K-slab of the CTA's first tile unfilled, so the
  // MMA issuer's wait for it runs out; -1 in every product launch.
  int stall_kb;
  // Split K (CTA-pair kernel, epilogues without EPI_POST, one destination):
  // work unit u of splits * tiles covers tile u % tiles over the K-slabs
  // [s * kb_split, min((s + 1) * kb_split, num_kb)), s = u / tiles; each
  // tile half's units meet in splitk_fixup.  splits == 1: one unit per
  // tile over the whole K range (the scratch pointers are unused).
  int splits;
  int kb_split;
  // Narrow last wave (CTA-pair kernel, plain epilogues): tiles [0,
  // narrow_first) run as one 256-column unit each; every later tile runs as
  // two 128-column units (M=256, N=128 MMAs), so a last wave that would
  // occupy at most half of the CTA pairs ends in about half a tile's time.
  // 0: every tile full width.
  int narrow_first;
  uint32_t* sk_count;  // [tiles][2] arrivals per tile half: zero on entry, left zero
  uint32_t* sk_ready;  // [splits - 1][tiles][2] partial slot written: zero on entry, left zero
  int32_t* sk_part;    // [splits - 1][tiles][2][128 rows][256 columns] int32 partials
  // Segmented rows (CTA-pair kernel, TMA stores; 0: off).  Logical row r of
  // A and of a_scale lies at row (r / a_seg) * a_seg_stride + a_seg_off of
  // the A / a_scale arrays (the A tensor map is then 3-D {K, a_seg,
  // M / a_seg} and encodes the stride and offset itself); logical output
  // row r at row r % o_seg of segment r / o_seg of the 3-D output tensor map
  // (which encodes that segment's place).  a_seg is a multiple of 128 and
  // o_seg of 32, so no TMA box straddles two segments; M is a multiple of
  // both.  Residual and gate rows stay logical.
  int a_seg;
  int64_t a_seg_stride, a_seg_off;
  int o_seg;
  int64_t o_seg_stride, o_seg_off;  // host side: the output tensor map's layout
};

// Memory row of logical A row r (segmented A, see GemmParams).
__device__ __forceinline__ int64_t a_mem_row(const GemmParams& p, int r) {
  if (p.a_seg == 0) return r;
  const int sg = r / p.a_seg;
  return (int64_t)sg * p.a_seg_stride + p.a_seg_off + (r - sg * p.a_seg);
}

// One 32 x 32 staged output box of logical rows row..row+31 to the output
// tensor map (2-D, or 3-D for segmented output rows).
__device__ __forceinline__ void store_out_box(const GemmParams& p, const CUtensorMap* tmC, const void* src, int x,
                                              int row) {
  if (p.o_seg == 0) {
    tma_store_2d(tmC, src, x, row);
  } else {
    const int sg = row / p.o_seg;
    tma_store_3d(tmC, src, x, row - sg * p.o_seg, sg);
  }
}

// Scratch layout of a split-K launch: a fixed header of counters and flags
// (the same place for every problem size, so one scratch buffer serves
// problems of any shape: every complete launch leaves the header zero),
// then the partial slots.
constexpr int SPLITK_MAX = 3;           // K parts per tile (the reader keeps SPLITK_MAX - 1 slots in flight)
constexpr int SPLITK_MAX_TILES = 2048;  // 256 x 256 tiles of a split problem
constexpr size_t SPLITK_HEADER = 65536;
struct SplitKLayout {
  size_t count_off, ready_off, part_off, bytes;
};
__host__ __device__ inline SplitKLayout splitk_layout(int tiles, int splits) {
  SplitKLayout l;
  l.count_off = 0;                                                   // [SPLITK_MAX_TILES][2]
  l.ready_off = (size_t)SPLITK_MAX_TILES * 2 * sizeof(uint32_t);     // [SPLITK_MAX - 1][tiles][2]
  l.part_off = SPLITK_HEADER;
  l.bytes = l.part_off + (size_t)(splits - 1) * tiles * 2 * 128 * 256 * sizeof(int32_t);
  return l;
}
static_assert((size_t)SPLITK_MAX_TILES * 2 * 4 * SPLITK_MAX <= SPLITK_HEADER, "split-K header");

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 128;  // bytes (= int8 elements) of K per stage
constexpr int EPI_WARPS = 8;  // epilogue warps (2 per TMEM lane quarter)

// Per-tile epilogue parameters (float weight scales and bias of the tile's
// columns), double-buffered by tile parity, in shared memory after the
// barriers.
template <int BN>
struct EpiSmem {
  float ws[2][BN];
  float bias[2][BN];
  float gate[2][BN];  // EPI_POST gate row of the tile (when its rows share one)
  int gate_ok[2];
  int sk_order;       // split K: this unit's arrival order on its tile half
};

template <int BN, bool B_INT4>
struct GemmCfg {
  static constexpr int STAGES = B_INT4 ? 3 : 4;
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK;
  static constexpr int B_BYTES = BN * GEMM_BK;
  static constexpr int BP_BYTES = B_INT4 ? BN * (GEMM_BK / 2) : 0;  // packed staging
  static constexpr int NUM_THREADS = B_INT4 ? 448 : 320;
  static constexpr int SMEM_BYTES = 1024 + STAGES * (A_BYTES + B_BYTES + BP_BYTES) + 256 + 16 + sizeof(EpiSmem<BN>);
  static constexpr uint32_t TMEM_COLS = 2 * BN;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  constexpr int GROUP_M = 8;
  const int per_group = GROUP_M * num_n;
  const int gid = tile / per_group;
  const int first_m = gid * GROUP_M;
  const int gsz = min(num_m - first_m, GROUP_M);
  const int in_g = tile % per_group;
  mb = first_m + in_g % gsz;
  nb = in_g / gsz;
}

// Units of a launch without split K: full tiles, then (narrow_first > 0)
// the remaining tiles as two 128-column units each.
__device__ __forceinline__ int full_or_narrow_units(const GemmParams& p, int num_tiles) {
  return p.narrow_first > 0 ? p.narrow_first + 2 * (num_tiles - p.narrow_first) : num_tiles;
}
// Unit u's row block, first column and width (columns) for BN-wide tiles.
template <int BN>
__device__ __forceinline__ int unit_geometry(const GemmParams& p, int u, int num_m, int num_n, int& mb, int& n0) {
  int nb;
  if (p.narrow_first == 0 || u < p.narrow_first) {
    tile_coords(u, num_m, num_n, mb, nb);
    n0 = nb * BN;
    return BN;
  }
  const int j = u - p.narrow_first;
  tile_coords(p.narrow_first + (j >> 1), num_m, num_n, mb, nb);
  n0 = nb * BN + (j & 1) * (BN / 2);
  return BN / 2;
}


template <int DT>
__device__ __forceinline__ void store_out_chunk(typename Elem<DT>::T* dst, const float (&y)[32], bool vec, int ncols) {
  if (vec) {
    if constexpr (DT == DT_F32) {
      float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
    } else {
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // values are already representable in DT: conversion is exact
        if constexpr (DT == DT_BF16) {
          __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
          w[j] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols) dst[j] = Elem<DT>::from_f(y[j]);
  }
}

// Unpack one packed-int4 K-slab (BN rows x 64 bytes, row-major, unswizzled)
// into the 128B-swizzled int8 layout TMA would have produced for an int8
// slab (16-byte chunk c of row r lands at chunk c ^ (r & 7)), each code q as
// the byte 16*q: the nibble moved to the high half of its byte needs no sign
// extension.  Consumers divide the products by 16 exactly (a power of two).
// Thread `tid` of NTHR handles rows tid/8 + k*NTHR/8, chunk tid%8: all its
// loads are issued before the first store, offsets are per-thread constants.
template <int BN, int NTHR>
__device__ __forceinline__ void unpack_int4_slab_x16(const uint8_t* src, uint8_t* dst, int tid) {
  static_assert(NTHR % 64 == 0 && (BN * 8) % NTHR == 0, "row step must keep r & 7");
  constexpr int ITEMS = BN * 8 / NTHR;
  constexpr int RSTEP = NTHR / 8;
  const int r0 = tid >> 3, c = tid & 7;
  const uint8_t* s0 = src + r0 * 64 + c * 8;
  uint8_t* d0 = dst + r0 * 128 + ((c ^ (r0 & 7)) << 4);
  uint2 pk[ITEMS];
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) pk[k] = *reinterpret_cast<const uint2*>(s0 + k * RSTEP * 64);
#pragma unroll
  for (int k = 0; k < ITEMS; ++k) {
    const uint32_t l0 = (pk[k].x << 4) & 0xF0F0F0F0u, h0 = pk[k].x & 0xF0F0F0F0u;
    const uint32_t l1 = (pk[k].y << 4) & 0xF0F0F0F0u, h1 = pk[k].y & 0xF0F0F0F0u;
    // interleave: k even <- low nibble, k odd <- high nibble
    *reinterpret_cast<uint4*>(d0 + k * RSTEP * 128) =
        make_uint4(__byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362), __byte_perm(l1, h1, 0x5140),
                   __byte_perm(l1, h1, 0x7362));
  }
}

// Per-tile epilogue parameters staged in shared memory by the epilogue warps
// one tile ahead (weight scales and bias of the tile's columns as float, and
// each thread's activation-row scale in a register), so no global load
// latency sits between the TMEM load and the stores.

// Named barrier among the 8 epilogue warps only.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(32 * EPI_WARPS) : "memory"); }

// Load this thread's share of a tile's per-column parameters (thread e of
// the epilogue handles column colt0 + e) into registers.
template <int BN, int EPI, int OUT_DT>
__device__ __forceinline__ void epi_load_params(const GemmParams& p, int colt0, int e, float& ws, float& b) {
  ws = 0.0f;
  b = 0.0f;
  if (e >= BN) return;
  const int col = colt0 + e;
  if (col >= p.N) return;
  if constexpr (epi_base(EPI) == EPI_W8A8_ROW) ws = __ldg(p.w_scale + col);
  // packed-int4 B is unpacked as 16*q: ws/16 (exact) restores the products
  if constexpr (epi_base(EPI) == EPI_W4A4_ROW) ws = __ldg(p.w_scale + col) * 0.0625f;
  if constexpr (EPI != EPI_I32) {
    if (p.bias != nullptr) b = Elem<OUT_DT>::to_f(reinterpret_cast<const typename Elem<OUT_DT>::T*>(p.bias)[col]);
  }
}

// tanh-form GELU, 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3),
// evaluated as the equal x * sigmoid(2u) = x / (1 + 2^(-2u log2(e))): the
// exponential and the reciprocal on the special-function unit (ex2.approx,
// rcp.approx; a few float32 units of error), so a 16-bit result is within
// one unit of the exact function's -- including where 1 + tanh(u) cancels
// in float32 (x < -3), which the tanh form evaluates with large relative
// error.  Infinities and NaN behave as in the tanh form (+inf -> +inf,
// -inf -> NaN, NaN -> NaN); large negative x gives -0.
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float kNeg2BetaLog2e = -2.302208198144325f;  // -2 sqrt(2/pi) / ln(2)
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float t = __fmul_rn(kNeg2BetaLog2e, __fmaf_rn(0.044715f, x3, x));
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(__fadd_rn(1.0f, e)));
  return __fmul_rn(x, r);
}

template <int DT>
__device__ __forceinline__ void unpack8(uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (DT == DT_BF16) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

// EPI_POST steps on one thread's 32 output columns [col0, col0 + ncols) of
// row `row` (values already rounded to the output dtype).  Residual and gate
// rows are 16-byte aligned (checked on the host).
template <int OUT_DT>
__device__ __forceinline__ void epi_post(const GemmParams& p, float (&y)[32], int row, int col0, int ncols) {
  using EO = Elem<OUT_DT>;
  using T = typename EO::T;
  if (p.gelu_col0 < (int64_t)col0 + 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j >= p.gelu_col0) y[j] = EO::round(gelu_tanh_f(y[j]));
  }
  if (p.residual == nullptr || row >= p.M) return;
  const T* rs = reinterpret_cast<const T*>(p.residual) + (int64_t)row * p.ld_res + col0;
  const T* gs = p.gate == nullptr ? nullptr
                                  : reinterpret_cast<const T*>(p.gate) + (int64_t)(row / p.rows_per_gate) * p.gate_ld + col0;
  if (ncols == 32) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float rv[8], gv[8];
      unpack8<OUT_DT>(__ldg(reinterpret_cast<const uint4*>(rs) + q), rv);
      if (gs != nullptr) {
        unpack8<OUT_DT>(__ldg(reinterpret_cast<const uint4*>(gs) + q), gv);
#pragma unroll
        for (int k = 0; k < 8; ++k) y[8 * q + k] = EO::round(__fadd_rn(rv[k], EO::round(__fmul_rn(gv[k], y[8 * q + k]))));
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) y[8 * q + k] = EO::round(__fadd_rn(rv[k], y[8 * q + k]));
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= ncols) continue;
      const float t = gs != nullptr ? EO::round(__fmul_rn(EO::to_f(gs[j]), y[j])) : y[j];
      y[j] = EO::round(__fadd_rn(EO::to_f(rs[j]), t));
    }
  }
}

// Epilogue of one 128-row accumulator tile held in TMEM columns
// [tmem_acc, tmem_acc + BN): this warp converts TMEM lane quarter `quarter`
// (rows row0 + 32*quarter + lane) and column half `half` (EPI_WARPS == 8),
// with the tile's per-column parameters in shared memory (s_ws, s_b).
// Stores through shared memory: each epilogue warp stages its 32 x 32 chunk
// of 16-bit outputs in a 2 KB buffer laid out with the 64-byte TMA swizzle
// (16-byte chunk k of row r at k ^ ((r >> 1) & 3): conflict-free row writes)
// and one lane issues a TMA tensor store of the box.
constexpr int EPI_STAGE_BYTES = 32 * 64;

template <int BN, int EPI, int OUT_DT, int ISHIFT>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, uint32_t tmem_acc, int row0, int colt0, int quarter,
                                              int half, int lane, const float* s_ws, const float* s_b, float xs,
                                              const CUtensorMap* tmC = nullptr, uint8_t* stage = nullptr) {
  using EO = Elem<OUT_DT>;  // EPI_I32 ignores it (instantiated with DT_F32)
  constexpr int EB = epi_base(EPI);
  constexpr bool POST = (EPI & EPI_POST) != 0;
  constexpr int CHUNKS = BN / 32;
  constexpr int CPW = CHUNKS / 2;  // chunks per warp
  const bool out16 = (OUT_DT == DT_BF16 || OUT_DT == DT_F16) && EB != EPI_I32;
  const int vec_n = out16 ? 8 : 4;
  // (every destination base is 16-byte aligned when nout > 1: checked on the host)
  const bool vec_ok = (p.ldo % vec_n) == 0 && (p.col_off % vec_n) == 0 &&
                      ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0);
  const bool has_bias = p.bias != nullptr;
  const int row = row0 + quarter * 32 + lane;
  const bool row_ok = row < p.M;
  float s_tensor = 0.0f;
  if constexpr (EB == EPI_W8A8_TENSOR) s_tensor = __fmul_rn(__ldg(p.w_scale), xs);
#pragma unroll 1
  for (int cc = 0; cc < CPW; ++cc) {
    const int c = half * CPW + cc;
    const int col0 = colt0 + c * 32;
    const int ncols = min(32, p.N - col0);
    const bool full_chunk = (ncols == 32) && vec_ok;
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem_acc + c * 32 + ((uint32_t)(quarter * 32) << 16), r);
    tmem_ld_wait();
    const bool tma_st = tmC != nullptr;  // warp-uniform
    // gathered (peer) outputs also go through the staging buffer, then leave
    // as row-contiguous stores
    const bool peer_st = !tma_st && stage != nullptr && p.nout > 1;
    const bool staged = tma_st || peer_st;
    if (staged ? (col0 >= p.N || row0 + quarter * 32 >= p.M) : (!row_ok || col0 >= p.N)) continue;
    if constexpr (EB == EPI_I32) {
      if constexpr (ISHIFT > 0) {
        // 16*q weights: the accumulator is 16x the product, exactly
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = (uint32_t)((int32_t)r[j] >> ISHIFT);
      }
      int32_t* dst = reinterpret_cast<int32_t*>(p.out) + (int64_t)row * p.ldo + p.col_off + col0;
      if (full_chunk) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          reinterpret_cast<int4*>(dst)[i] = make_int4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < ncols) dst[j] = (int32_t)r[j];
      }
    } else {
      const float4* w4 = reinterpret_cast<const float4*>(s_ws + c * 32);
      const float4* b4 = reinterpret_cast<const float4*>(s_b + c * 32);
      float y[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float wv[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (EB != EPI_W8A8_TENSOR) {
          const float4 t = w4[i];
          wv[0] = t.x; wv[1] = t.y; wv[2] = t.z; wv[3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = 4 * i + k;
          const float f = __int2float_rn((int32_t)r[j]);  // res.float()
          float v;
          if constexpr (EB == EPI_W8A8_TENSOR) {
            v = EO::round(__fmul_rn(f, s_tensor));             // .mul_(ws * xs).to(dt)
          } else if constexpr (EB == EPI_W8A8_ROW) {
            v = EO::round(__fmul_rn(__fmul_rn(f, xs), wv[k]));  // .mul_(xs).mul_(ws.T).to(dt)
          } else {
            v = __fmul_rn(__fmul_rn(f, xs), wv[k]);            // float32, rounded once below
          }
          y[j] = v;
        }
      }
      if (has_bias) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 t = b4[i];
          y[4 * i] = EO::round(__fadd_rn(y[4 * i], t.x));
          y[4 * i + 1] = EO::round(__fadd_rn(y[4 * i + 1], t.y));
          y[4 * i + 2] = EO::round(__fadd_rn(y[4 * i + 2], t.z));
          y[4 * i + 3] = EO::round(__fadd_rn(y[4 * i + 3], t.w));
        }
      } else if constexpr (EB == EPI_W4A4_ROW) {
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = EO::round(y[j]);
      }
      if constexpr (POST) epi_post<OUT_DT>(p, y, row, col0, ncols);
      if constexpr (OUT_DT == DT_BF16 || OUT_DT == DT_F16) {
        if (staged) {
          uint32_t w[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if constexpr (OUT_DT == DT_BF16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
              w[j] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
              w[j] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          if (tma_st && lane == 0) bulk_wait_read_all();  // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 4; ++k)
            *reinterpret_cast<uint4*>(stage + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          if (tma_st) {
            fence_proxy_async_smem();  // generic-proxy writes -> TMA reads
            __syncwarp();
            if (lane == 0) {
              store_out_box(p, tmC, stage, (int)(p.col_off + col0), row0 + quarter * 32);
              bulk_commit_group();
            }
            continue;
          }
          __syncwarp();
          // 128 16-byte granules (32 rows x 4): lane l takes granules l, l+32,
          // l+64, l+96, so each store instruction covers 8 whole row segments
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int g = lane + 32 * it;
            const int rr = g >> 2, k = g & 3;
            const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 64 + ((k ^ ((rr >> 1) & 3)) << 4));
            const int grow = row0 + quarter * 32 + rr;
            const int gcol = col0 + 8 * k;
            if (grow >= p.M || gcol >= p.N) continue;
            const int64_t off = (int64_t)grow * p.ldo + p.col_off + gcol;
            if (gcol + 8 <= p.N) {
              for (int o = 0; o < p.nout; ++o)
                *reinterpret_cast<uint4*>(reinterpret_cast<typename EO::T*>(p.outs[o]) + off) = v;
            } else {
              const typename EO::T* e = reinterpret_cast<const typename EO::T*>(&v);
              for (int o = 0; o < p.nout; ++o)
                for (int j = 0; j < p.N - gcol; ++j) reinterpret_cast<typename EO::T*>(p.outs[o])[off + j] = e[j];
            }
          }
          __syncwarp();  // staging buffer reused by the next chunk
          continue;
        }
      }
      const int64_t off = (int64_t)row * p.ldo + p.col_off + col0;
      if (p.nout == 1) {
        store_out_chunk<OUT_DT>(reinterpret_cast<typename EO::T*>(p.out) + off, y, full_chunk, ncols);
      } else {
        // tensor-parallel gather: the same chunk into every rank's buffer
        for (int o = 0; o < p.nout; ++o)
          store_out_chunk<OUT_DT>(reinterpret_cast<typename EO::T*>(p.outs[o]) + off, y, full_chunk, ncols);
      }
    }
  }
}

// Residual values of row `row`, columns [col0, col0 + 32) of an EPI_POST
// residual, as 16 packed pairs (zeros outside the tensor).  Rows are 16-byte
// aligned (checked on the host).
template <int OUT_DT>
__device__ __forceinline__ void load_res32(const GemmParams& p, int row, int col0, uint4 (&rv)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) rv[q] = make_uint4(0u, 0u, 0u, 0u);
  if (p.residual == nullptr || row < 0 || row >= p.M || col0 >= p.N) return;
  const uint16_t* rs = reinterpret_cast<const uint16_t*>(p.residual) + (int64_t)row * p.ld_res + col0;
  if (col0 + 32 <= p.N) {
#pragma unroll
    for (int q = 0; q < 4; ++q) rv[q] = __ldg(reinterpret_cast<const uint4*>(rs) + q);
  } else {
    const int n = p.N - col0;
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const uint32_t lo = 2 * j < n ? (uint32_t)rs[2 * j] : 0u;
      const uint32_t hi = 2 * j + 1 < n ? (uint32_t)rs[2 * j + 1] : 0u;
      w[j] = lo | (hi << 16);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) rv[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
}

// Round 32 float values to the 16-bit dtype and back, two per conversion
// instruction (cvt.rn.{bf16x2,f16x2}.f32): the conversion unit, which
// handles 16 operations per clock per SM, bounds this epilogue, so every
// rounding step goes through it in pairs.
template <int OUT_DT>
__device__ __forceinline__ void rnd_pairs(float (&y)[32]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (OUT_DT == DT_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
      const uint32_t u = *reinterpret_cast<uint32_t*>(&h);
      y[2 * j] = __uint_as_float(u << 16);
      y[2 * j + 1] = __uint_as_float(u & 0xFFFF0000u);
    } else {
      const float2 f = __half22float2(__floats2half2_rn(y[2 * j], y[2 * j + 1]));
      y[2 * j] = f.x;
      y[2 * j + 1] = f.y;
    }
  }
}

// One 32-column chunk of the TMA-store epilogue: accumulator registers `r`
// (already waited for) -> the reference's epilogue -> EPI_POST steps ->
// 16-bit values staged in `sb` (64-byte TMA swizzle) -> one TMA store.
// `g32`: the tile's gate row staged in shared memory, or null (per-row gate
// loads).  With EPI_POST the bulk stores are double-buffered per warp:
// before `sb` is written, every store but the most recent one (which used
// the other buffer) has read its source; otherwise one buffer, free once the
// previous store has read it.
template <int EPI, int OUT_DT>
__device__ __forceinline__ void epi_chunk_tma(const GemmParams& p, const uint32_t (&r)[32], const uint4 (&rv)[4],
                                              const float* ws32, const float* b32, const float* g32, float xs,
                                              float s_tensor, bool has_bias, int row, int row_base, int col0, int lane,
                                              const CUtensorMap* tmC, uint8_t* sb) {
  constexpr int EB = epi_base(EPI);
  constexpr bool POST = (EPI & EPI_POST) != 0;
  // The reference's rounding sequence with each dt() applied in pairs; the
  // last dt() of the chain is the packing conversion of the store, so a
  // value is never converted twice:
  //   W8A8: dt(dt(float(acc) * xs * ws) + bias)   W4A4: dt(float(acc) * xs * ws + bias)
  float y[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float wv[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (EB != EPI_W8A8_TENSOR) {
      const float4 t = reinterpret_cast<const float4*>(ws32)[i];
      wv[0] = t.x; wv[1] = t.y; wv[2] = t.z; wv[3] = t.w;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 4 * i + k;
      const float f = __int2float_rn((int32_t)r[j]);  // res.float()
      if constexpr (EB == EPI_W8A8_TENSOR) {
        y[j] = __fmul_rn(f, s_tensor);              // .mul_(ws * xs)
      } else {
        y[j] = __fmul_rn(__fmul_rn(f, xs), wv[k]);  // .mul_(xs).mul_(ws.T)
      }
    }
  }
  if constexpr (EB != EPI_W4A4_ROW) rnd_pairs<OUT_DT>(y);  // .to(dt)
  if (has_bias) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = reinterpret_cast<const float4*>(b32)[i];
      y[4 * i] = __fadd_rn(y[4 * i], t.x);
      y[4 * i + 1] = __fadd_rn(y[4 * i + 1], t.y);
      y[4 * i + 2] = __fadd_rn(y[4 * i + 2], t.z);
      y[4 * i + 3] = __fadd_rn(y[4 * i + 3], t.w);
    }
  }
  if constexpr (POST) {
    // the steps below take the dtype value of the linear's output
    if (has_bias || EB == EPI_W4A4_ROW) rnd_pairs<OUT_DT>(y);
    if (p.gelu_col0 <= (int64_t)col0) {
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = gelu_tanh_f(y[j]);
      if (p.residual != nullptr) rnd_pairs<OUT_DT>(y);
    } else if (p.gelu_col0 < (int64_t)col0 + 32) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j >= p.gelu_col0) y[j] = gelu_tanh_f(y[j]);
      rnd_pairs<OUT_DT>(y);  // exact on the columns that were already rounded
    }
    if (p.residual != nullptr) {
      float rres[32];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float t8[8];
        unpack8<OUT_DT>(rv[q], t8);
#pragma unroll
        for (int k = 0; k < 8; ++k) rres[8 * q + k] = t8[k];
      }
      if (p.gate != nullptr) {
        float gv[32];
        if (g32 != nullptr) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 t = reinterpret_cast<const float4*>(g32)[i];
            gv[4 * i] = t.x; gv[4 * i + 1] = t.y; gv[4 * i + 2] = t.z; gv[4 * i + 3] = t.w;
          }
        } else {
          // the CTA's rows span two gate rows: this row's own gate values
          const uint16_t* gs = reinterpret_cast<const uint16_t*>(p.gate) +
                               (int64_t)(min(row, p.M - 1) / p.rows_per_gate) * p.gate_ld + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const uint16_t h = col0 + j < p.N ? gs[j] : (uint16_t)0;
            if constexpr (OUT_DT == DT_BF16) gv[j] = __uint_as_float((uint32_t)h << 16);
            else gv[j] = __half2float(__ushort_as_half(h));
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) y[j] = __fmul_rn(gv[j], y[j]);
        rnd_pairs<OUT_DT>(y);  // dt(gate * y)
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) y[j] = __fadd_rn(rres[j], y[j]);  // rounded by the store's packing
    }
  }
  uint32_t w[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if constexpr (OUT_DT == DT_BF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * j], y[2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    } else {
      __half2 h = __floats2half2_rn(y[2 * j], y[2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
  if (lane == 0) {
    if constexpr (POST) bulk_wait_read_1();  // the store two chunks back (same buffer) has read it
    else bulk_wait_read_all();               // one buffer: the previous store has read it
  }
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *reinterpret_cast<uint4*>(sb + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
        make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  fence_proxy_async_smem();  // generic-proxy writes -> TMA reads
  __syncwarp();
  if (lane == 0) {
    store_out_box(p, tmC, sb, (int)(p.col_off + col0), row_base);
    bulk_commit_group();
  }
}

// Epilogue of one 128-row accumulator tile for 16-bit outputs leaving
// through TMA stores (one destination).  With EPI_POST, stores alternate
// between the warp's two staging buffers (`stc` counts this warp's stores
// across tiles and picks the buffer).  Without EPI_POST the warp's CPW chunks are
// software pipelined: the TMEM load of chunk c+1 is in flight while chunk c
// is converted and stored.  With EPI_POST (register budget: one accumulator
// chunk at a time) the residual loads of chunk c+1 are in flight instead;
// `res` holds the residual of the warp's first chunk on entry (loaded
// during the previous tile) and of the next tile's first chunk (row `nrow`,
// column `ncol0`; nrow < 0: none) on return.
template <int BN, int EPI, int OUT_DT>
__device__ __forceinline__ void epilogue_tile_tma(const GemmParams& p, uint32_t tmem_acc, int row0, int colt0,
                                                  int quarter, int half, int lane, const float* s_ws,
                                                  const float* s_b, const float* s_gate, float xs,
                                                  const CUtensorMap* tmC, uint8_t* stage, uint32_t& stc,
                                                  uint4 (&res)[4], int nrow, int ncol0) {
  constexpr int EB = epi_base(EPI);
  constexpr bool POST = (EPI & EPI_POST) != 0;
  constexpr int CPW = BN / 64;  // chunks per warp (two warps per lane quarter)
  static_assert(CPW % 2 == 0, "chunks are processed in pairs");
  const bool has_bias = p.bias != nullptr;
  const int row = row0 + quarter * 32 + lane;
  const int row_base = row0 + quarter * 32;
  float s_tensor = 0.0f;
  if constexpr (EB == EPI_W8A8_TENSOR) s_tensor = __fmul_rn(__ldg(p.w_scale), xs);
  const int c0 = half * CPW;
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const bool quarter_live = row_base < p.M;  // warp-uniform
  if constexpr (POST) {
    const bool has_res = p.residual != nullptr;
#pragma unroll 1
    for (int cc = 0; cc < CPW; ++cc) {
      const int col = colt0 + (c0 + cc) * 32;
      uint32_t ra[32];
      tmem_ld_32x32b_x32(tmem_acc + (c0 + cc) * 32 + lane_off, ra);
      uint4 rn[4];
      if (has_res) {
        if (cc + 1 < CPW) load_res32<OUT_DT>(p, row, col + 32, rn);
        else load_res32<OUT_DT>(p, nrow < 0 ? -1 : nrow, ncol0, rn);  // the next tile's first chunk
      }
      tmem_ld_wait_regs(ra);
      if (quarter_live && col < p.N) {
        epi_chunk_tma<EPI, OUT_DT>(p, ra, res, s_ws + (c0 + cc) * 32, s_b + (c0 + cc) * 32,
                                   s_gate ? s_gate + (c0 + cc) * 32 : nullptr, xs, s_tensor, has_bias, row, row_base,
                                   col, lane, tmC, stage + (stc & 1) * EPI_STAGE_BYTES);
        ++stc;
      }
      if (has_res) {
#pragma unroll
        for (int q = 0; q < 4; ++q) res[q] = rn[q];
      }
    }
    return;
  }
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(tmem_acc + c0 * 32 + lane_off, ra);
#pragma unroll 1
  for (int cc = 0; cc < CPW; cc += 2) {
    const int colA = colt0 + (c0 + cc) * 32;
    const int colB = colA + 32;
    tmem_ld_wait_regs(ra);
    tmem_ld_32x32b_x32(tmem_acc + (c0 + cc + 1) * 32 + lane_off, rb);
    if (quarter_live && colA < p.N) {
      epi_chunk_tma<EPI, OUT_DT>(p, ra, res, s_ws + (c0 + cc) * 32, s_b + (c0 + cc) * 32, nullptr, xs, s_tensor,
                                 has_bias, row, row_base, colA, lane, tmC, stage);
      ++stc;
    }
    tmem_ld_wait_regs(rb);
    if (cc + 2 < CPW) tmem_ld_32x32b_x32(tmem_acc + (c0 + cc + 2) * 32 + lane_off, ra);
    if (quarter_live && colB < p.N) {
      epi_chunk_tma<EPI, OUT_DT>(p, rb, res, s_ws + (c0 + cc + 1) * 32, s_b + (c0 + cc + 1) * 32, nullptr, xs,
                                 s_tensor, has_bias, row, row_base, colB, lane, tmC,
                                 stage);
      ++stc;
    }
  }
}

// 32 lanes x 16 columns of 32-bit TMEM -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// tcgen05.wait::ld tied to the 16 registers of one tmem_ld_32x32b_x16.
__device__ __forceinline__ void tmem_ld_wait_regs16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}
// 32 lanes x 16 columns of 32-bit TMEM <- 16 registers per thread.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// 32 lanes x 32 columns of 32-bit TMEM <- 32 registers per thread.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* a, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// Split K: the units of one tile half (this CTA's 128 rows of a 256 x 256
// tile) meet here after their MMAs, all 8 epilogue warps of the CTA taking
// part.  The arrival order comes from an atomic counter (one per tile half):
// units 0 .. splits-2 store their int32 accumulator in their own scratch
// slot and publish it with a release flag; the last unit waits (bounded)
// for those flags, adds the slots into its accumulator in TMEM (int32
// additions: exact, so the result does not depend on which unit is last)
// and returns true -- it runs the tile's normal epilogue -- after putting
// the counter and flags back to zero for the next launch.  The waits are on
// units that have already arrived, i.e. are past their MMAs and storing.
// A slot holds each epilogue warp's 32 x 128 block as [chunk][quad][lane]
// 16-byte vectors, so every warp-wide access is 512 contiguous bytes.
template <int BN>
__device__ __forceinline__ bool splitk_fixup(const GemmParams& p, EpiSmem<BN>* es, volatile int* abort_flag,
                                             uint32_t tmem_acc, int tile, int num_tiles, int rank, int warp,
                                             int lane) {
  static_assert(BN == 256, "CTA-pair tiles");
  const int e = (warp - 2) * 32 + lane;  // 0..255
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const int slot = tile * 2 + rank;  // this tile half
  const int last = p.splits - 1;
  if (e == 0) {
    const uint32_t o = atomicAdd(&p.sk_count[slot], 1u);
    if (o > (uint32_t)last) {  // the counters were not zero on entry: refuse, report
      atomicOr(&g_error_bits, 8u);
      *abort_flag = 1;
    }
    es->sk_order = (int)o;
  }
  epi_bar();
  if (*abort_flag) return false;
  const int order = es->sk_order;
  // this warp's 32 x 128 block in slot j: 4 chunks x 8 quads x 32 lanes of int4
  auto block = [&](int j) {
    return reinterpret_cast<int4*>(p.sk_part) + (((size_t)j * num_tiles * 2 + slot) * 8 + (half * 4 + quarter)) * 1024;
  };
  if (order < last) {
    int4* dst = block(order);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tmem_acc + (uint32_t)(half * 128 + c * 32) + lane_off, r);
      tmem_ld_wait_regs(r);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        __stcg(dst + (c * 8 + q) * 32 + lane,
               make_int4((int)r[4 * q], (int)r[4 * q + 1], (int)r[4 * q + 2], (int)r[4 * q + 3]));
    }
    epi_bar();  // every warp's stores precede the flag
    if (e == 0) {
      __threadfence();
      st_release_gpu(&p.sk_ready[(size_t)order * num_tiles * 2 + slot], 1u);
    }
    return false;
  }
  if (e == 0) {
    const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
    const uint64_t t0 = globaltimer_ns();
    for (int j = 0; j < last && !*abort_flag; ++j) {
      const uint32_t* f = &p.sk_ready[(size_t)j * num_tiles * 2 + slot];
      uint32_t iter = 0;
      while (ld_acquire_gpu(f) == 0u) {
        if ((++iter & 63u) == 0) {
          if (*abort_flag) break;
          if (globaltimer_ns() - t0 > limit) {
            atomicOr(&g_error_bits, 1u);
            *abort_flag = 1;
            break;
          }
        }
      }
    }
  }
  epi_bar();
  if (*abort_flag) return false;
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {  // 16-column sub-chunks: quads 4 * (c & 1) .. of chunk c >> 1
    const uint32_t ta = tmem_acc + (uint32_t)(half * 128 + c * 16) + lane_off;
    uint32_t r[16];
    tmem_ld_32x32b_x16(ta, r);
    int4 v[SPLITK_MAX - 1][4];  // every slot's quads in flight at once
#pragma unroll
    for (int j = 0; j < SPLITK_MAX - 1; ++j)
      if (j < last) {
        const int4* src = block(j) + ((c >> 1) * 8 + 4 * (c & 1)) * 32 + lane;
#pragma unroll
        for (int q = 0; q < 4; ++q) v[j][q] = __ldcg(src + q * 32);
      }
    tmem_ld_wait_regs16(r);
#pragma unroll
    for (int j = 0; j < SPLITK_MAX - 1; ++j)
      if (j < last) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          r[4 * q] += (uint32_t)v[j][q].x;
          r[4 * q + 1] += (uint32_t)v[j][q].y;
          r[4 * q + 2] += (uint32_t)v[j][q].z;
          r[4 * q + 3] += (uint32_t)v[j][q].w;
        }
      }
    tmem_st_32x32b_x16(ta, r);
  }
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
  if (e == 0) {  // every unit of this tile half has arrived: reset for the next launch
    p.sk_count[slot] = 0u;
    for (int j = 0; j < last; ++j) p.sk_ready[(size_t)j * num_tiles * 2 + slot] = 0u;
  }
  return true;
}

// The epilogue role of a GEMM kernel: for each tile of this CTA, wait for the
// accumulator, convert it, release it.  Parameters of tile i+1 are loaded into
// registers while tile i is converted and staged into shared memory after it.
// All epilogue threads pass the named barrier every tile and leave together
// when any wait timed out (the abort flag is read after the barrier).
template <int BN, int EPI, int OUT_DT, int ROWS_PER_TILE, bool PAIR, int ISHIFT = 0, bool SPLIT = false>
__device__ __forceinline__ void epilogue_role(const GemmParams& p, EpiSmem<BN>* es, uint64_t* tfull, uint64_t* tempty,
                                              volatile int* abort_flag, uint32_t tmem_base, int first_tile,
                                              int tile_stride, int num_tiles, int num_m, int num_n, int row_off,
                                              int warp, int lane, const CUtensorMap* tmC = nullptr,
                                              uint8_t* stage = nullptr) {
  const int e = (warp - 2) * 32 + lane;  // 0..255
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  constexpr bool TMA16 = (OUT_DT == DT_BF16 || OUT_DT == DT_F16) && EPI != EPI_I32;
  constexpr bool POST = (EPI & EPI_POST) != 0;
  constexpr int CPW = BN / 64;
  int acc = 0;
  uint32_t acc_phase = 0;
  float nws, nb, nxs = 0.0f, ngate = 0.0f;
  int ngok = 0;
  int buf = 0;
  uint32_t stc = 0;  // TMA stores issued by this warp (staging buffer parity)
  uint4 res[4] = {};
  // EPI_POST gate of a tile: staged when the CTA's rows of the tile share one
  // gate row (warp-uniform), else read per row in the epilogue
  auto load_gate = [&](int mb, int n0, float& g, int& ok) {
    g = 0.0f;
    ok = 0;
    if constexpr (POST) {
      if (p.gate == nullptr || p.residual == nullptr) return;
      const int r_first = mb * ROWS_PER_TILE + row_off;
      if (r_first >= p.M) return;
      const int r_last = min(r_first + GEMM_BM - 1, p.M - 1);
      if ((int64_t)r_first / p.rows_per_gate != (int64_t)r_last / p.rows_per_gate) return;
      ok = 1;
      const int col = n0 + e;
      if (e < BN && col < p.N) {
        const uint16_t h =
            reinterpret_cast<const uint16_t*>(p.gate)[((int64_t)r_first / p.rows_per_gate) * p.gate_ld + col];
        g = OUT_DT == DT_BF16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
      }
    }
  };
  // EPI_POST residual rows of a tile (this lane's row, the warp's columns)
  // into L2 a tile ahead of their use
  auto prefetch_res = [&](int mb, int n0) {
    if constexpr (TMA16 && POST) {
      if (tmC == nullptr || p.residual == nullptr) return;
      const int row = mb * ROWS_PER_TILE + row_off + quarter * 32 + lane;
      const int col0 = n0 + half * CPW * 32;
      if (row >= p.M || col0 >= p.N) return;
      const uint32_t bytes = (uint32_t)(min(CPW * 32, p.N - col0) * 2) & ~15u;
      if (bytes) bulk_prefetch_l2(reinterpret_cast<const uint16_t*>(p.residual) + (int64_t)row * p.ld_res + col0, bytes);
    }
  };
  // split K (pair kernel): work units cycle over the tiles once per split
  static_assert(!SPLIT || (PAIR && !POST), "split K: CTA-pair kernel, plain epilogues");
  // unit u: its tile, row block, first column and width (split K: whole
  // tiles, u cycling over them once per split; else see unit_geometry)
  const int num_units = SPLIT ? num_tiles * p.splits : full_or_narrow_units(p, num_tiles);
  auto geometry = [&](int u, int& mb, int& n0) {
    if constexpr (SPLIT) {
      int nbt;
      tile_coords(u % num_tiles, num_m, num_n, mb, nbt);
      n0 = nbt * BN;
      return BN;
    } else {
      return unit_geometry<BN>(p, u, num_m, num_n, mb, n0);
    }
  };
  if (first_tile < num_units) {
    int mb, n0_;
    geometry(first_tile, mb, n0_);
    prefetch_res(mb, n0_);
    epi_load_params<BN, EPI, OUT_DT>(p, n0_, e, nws, nb);
    const int row = mb * ROWS_PER_TILE + row_off + quarter * 32 + lane;
    if constexpr (EPI != EPI_I32) nxs = row < p.M ? __ldg(p.a_scale + a_mem_row(p, row)) : 0.0f;
    load_gate(mb, n0_, ngate, ngok);
    if (e < BN) { es->ws[0][e] = nws; es->bias[0][e] = nb; es->gate[0][e] = ngate; }
    if (e == 0) es->gate_ok[0] = ngok;
    if constexpr (TMA16 && POST) {
      if (tmC != nullptr && p.residual != nullptr) load_res32<OUT_DT>(p, row, n0_ + half * CPW * 32, res);
    }
  }
  for (int u = first_tile; u < num_units; u += tile_stride) {
    const int tile = u % num_tiles;  // split K only
    int mb, n0;
    const int width = geometry(u, mb, n0);
    // a narrow unit's columns are the first half: the second-half warps
    // store nothing (they still take part in every barrier and arrival)
    const bool idle_half = half * (BN / 2) >= width;
    const float xs = nxs;
    mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag);
    epi_bar();
    if (*abort_flag) break;
    tc_fence_after();
    const bool has_next = u + tile_stride < num_units;
    int nrow = -1, ncol0 = 0;
    if (has_next) {
      int mb2, n02;
      geometry(u + tile_stride, mb2, n02);
      epi_load_params<BN, EPI, OUT_DT>(p, n02, e, nws, nb);
      const int row = mb2 * ROWS_PER_TILE + row_off + quarter * 32 + lane;
      if constexpr (EPI != EPI_I32) nxs = row < p.M ? __ldg(p.a_scale + a_mem_row(p, row)) : 0.0f;
      load_gate(mb2, n02, ngate, ngok);
      prefetch_res(mb2, n02);
      nrow = row;
      ncol0 = n02 + half * CPW * 32;
    }
    bool done = false;
    if constexpr (SPLIT) {
      // split K: only the last unit of this tile half converts and stores
      done = !splitk_fixup<BN>(p, es, abort_flag, tmem_base + acc * BN, tile, num_tiles, row_off / GEMM_BM, warp,
                                 lane);
    }
    if (idle_half) done = true;  // narrow unit (plain epilogues only: no residual pipeline to keep)
    if constexpr (TMA16) {
      if (tmC != nullptr && !done) {
        epilogue_tile_tma<BN, EPI, OUT_DT>(p, tmem_base + acc * BN, mb * ROWS_PER_TILE + row_off, n0, quarter,
                                           half, lane, es->ws[buf], es->bias[buf],
                                           es->gate_ok[buf] ? es->gate[buf] : nullptr, xs, tmC, stage, stc, res,
                                           nrow, ncol0);
        done = true;
      }
    }
    if (!done)
      epilogue_tile<BN, EPI, OUT_DT, ISHIFT>(p, tmem_base + acc * BN, mb * ROWS_PER_TILE + row_off, n0, quarter,
                                             half, lane, es->ws[buf], es->bias[buf], xs, tmC, stage);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if constexpr (PAIR) {
        mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      } else {
        mbar_arrive(&tempty[acc]);
      }
    }
    buf ^= 1;
    if (has_next && e < BN) { es->ws[buf][e] = nws; es->bias[buf][e] = nb; es->gate[buf][e] = ngate; }
    if (has_next && e == 0) es->gate_ok[buf] = ngok;
    acc ^= 1;
    if (acc == 0) acc_phase ^= 1;
  }
  // peer stores are made visible system-wide before the kernel ends (the
  // caller's cross-GPU barrier orders them with the peers' reads)
  if (p.nout > 1) __threadfence_system();
  if (tmC != nullptr && lane == 0) bulk_wait_all();  // TMA stores complete before exit
}

template <int BN, int EPI, int OUT_DT, bool B_INT4>
__global__ void __launch_bounds__(GemmCfg<BN, B_INT4>::NUM_THREADS, 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   GemmParams p) {
  using Cfg = GemmCfg<BN, B_INT4>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* sBP = sB + STAGES * Cfg::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sBP + STAGES * Cfg::BP_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;      // B unpacked and ready (B_INT4)
  uint64_t* tfull = conv + STAGES;      // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* drain = tempty + 2;         // abort path: the MMA issuer's last commit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);  // 4 converter warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    mbar_init(drain, 1);
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

  const int num_m = (p.M + GEMM_BM - 1) / GEMM_BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + GEMM_BK - 1) / GEMM_BK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      ArmedLoads armed;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          if (!(kb == p.stall_kb && tile == (int)blockIdx.x)) {
            if constexpr (B_INT4) {
              mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::BP_BYTES);
              tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, mb * GEMM_BM);
              tma_load_2d(sBP + stage * Cfg::BP_BYTES, &tmB, &full[stage], kb * (GEMM_BK / 2), nb * BN);
            } else {
              mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::B_BYTES);
              tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, mb * GEMM_BM);
              tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * GEMM_BK, nb * BN);
            }
            armed.note(stage, phase);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      armed.drain(full, STAGES);  // no load still writing shared memory at exit
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(GEMM_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false, ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if constexpr (B_INT4) {
            if (!mbar_wait_bounded(&conv[stage], phase, abort_flag)) { ok = false; break; }
          } else {
            if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_k_sw128(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bdesc = umma_desc_k_sw128(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 32; ++k) {
            // advance 32 bytes of K inside the 128-byte swizzle atom
            umma_i8(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
          }
          issued = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (*abort_flag && issued) {  // MMAs complete before TMEM is released
        umma_commit(drain);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (warp < 2 + EPI_WARPS) {
    // ---------------- epilogue ----------------
    EpiSmem<BN>* es = reinterpret_cast<EpiSmem<BN>*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));
    epilogue_role<BN, EPI, OUT_DT, GEMM_BM, false, B_INT4 ? 4 : 0>(p, es, tfull, tempty, abort_flag, tmem_base, blockIdx.x, gridDim.x,
                                                   num_tiles, num_m, num_n, 0, warp, lane);
  } else if constexpr (B_INT4) {
    // ---------------- int4 -> int8 converters (warps 10..13) ----------------
    const int ctid = threadIdx.x - 32 * (2 + EPI_WARPS);
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
        unpack_int4_slab_x16<BN, 128>(sBP + stage * Cfg::BP_BYTES, sB + stage * Cfg::B_BYTES, ctid);
        fence_proxy_async_smem();  // generic-proxy writes -> tensor-core reads
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
// CTA-pair variant (cta_group::2): a 2-CTA cluster computes a 256 x 256 tile.
// Each CTA TMA-loads its own 128 rows of A and its own 128 rows of B (no
// multicast loads); the leader's single MMA thread issues M=256, N=256
// tcgen05.mma that read both CTAs' shared memory, each CTA's TMEM receiving
// its 128 output rows.  Per SM this streams 32 KB per 128-deep K step
// instead of 48 KB, so the L2 feed keeps up with the tensor cores.
//   full[s]   leader only: one expect_tx arrival (both CTAs' bytes)
//   empty[s]  both CTAs: the leader's commit multicasts to the pair
//   tfull[b]  both CTAs: multicast commit at tile end
//   tempty[b] leader only: 8 local + 8 remote epilogue-warp arrivals
// ---------------------------------------------------------------------------
template <int EPI, int OUT_DT, bool B_INT4 = false>
struct PairCfg {
  static constexpr int BN = 256;           // tile columns (both CTAs)
  static constexpr int BNH = 128;          // B rows loaded per CTA
  // 16-bit outputs leave through TMA stores staged per epilogue warp in 2 KB
  // buffers: one, or two with the EPI_POST steps (whose longer epilogue
  // overlaps a store with the next chunk; the operand ring gives up a stage)
  static constexpr bool TMA_ST = (OUT_DT == DT_BF16 || OUT_DT == DT_F16) && EPI != EPI_I32;
  static constexpr int EPI_BUFS = (EPI & EPI_POST) ? 2 : 1;
  // packed-int4 B: each CTA also stages its 128 packed weight rows (8 KB)
  // per K slab and two unpack warps (after the epilogue warps) expand them
  static constexpr int STAGES = B_INT4 ? 5 : ((TMA_ST && EPI_BUFS == 2) ? 5 : 6);
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK;   // 16 KB
  static constexpr int B_BYTES = BNH * GEMM_BK;       // 16 KB
  static constexpr int BP_BYTES = B_INT4 ? BNH * GEMM_BK / 2 : 0;  // 8 KB packed
  static constexpr int UNPACK_WARPS = B_INT4 ? 2 : 0;
  static constexpr int NUM_THREADS = 32 * (2 + EPI_WARPS + UNPACK_WARPS);
  static constexpr int STAGE_BYTES = TMA_ST ? EPI_WARPS * EPI_BUFS * EPI_STAGE_BYTES : 0;
  static constexpr int SMEM_BYTES =
      1024 + STAGES * (A_BYTES + B_BYTES + BP_BYTES) + STAGE_BYTES + 256 + 16 + sizeof(EpiSmem<BN>);
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory");
  static_assert(3 * STAGES * 8 + 4 * 8 + 8 + 8 <= 256, "barrier block");
  static constexpr uint32_t TMEM_COLS = 2 * BN;
};

// Nibble unpack of 64 rows of packed int4 (64 bytes of K each) into the
// 128-byte swizzled int8 layout (16*q per byte), rows 64*part.. of a
// 128-row slab, by one warp.
__device__ __forceinline__ void unpack_int4_rows64_warp(const uint8_t* src, uint8_t* dst, int part, int lane) {
  const int c = lane & 7;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint2 pk[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = 64 * part + (lane >> 3) + 4 * (8 * h + k);
      pk[k] = *reinterpret_cast<const uint2*>(src + row * 64 + c * 8);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = 64 * part + (lane >> 3) + 4 * (8 * h + k);
      const uint32_t l0 = (pk[k].x << 4) & 0xF0F0F0F0u, h0 = pk[k].x & 0xF0F0F0F0u;
      const uint32_t l1 = (pk[k].y << 4) & 0xF0F0F0F0u, h1 = pk[k].y & 0xF0F0F0F0u;
      *reinterpret_cast<uint4*>(dst + row * 128 + ((c ^ (row & 7)) << 4)) =
          make_uint4(__byte_perm(l0, h0, 0x5140), __byte_perm(l0, h0, 0x7362), __byte_perm(l1, h1, 0x5140),
                     __byte_perm(l1, h1, 0x7362));
    }
  }
}

// tmC: the output as a 16-bit 2-D tensor map with 32 x 32 boxes and the
// 64-byte swizzle; used when `use_tma_store` (one 16-byte-aligned
// destination), else the epilogue stores directly.
// B_INT4: B is packed int4 [N, K/2]; each CTA TMA-loads its 128 packed rows
// with its activation rows onto its own `full` barrier, its two unpack warps
// expand them and arrive on the leader's `conv` barrier (remotely, with
// CTA-scope release, from the peer), and the MMA waits on `conv`.
template <int EPI, int OUT_DT, bool SPLIT = false, bool B_INT4 = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<EPI, OUT_DT, B_INT4>::NUM_THREADS, 1)
    gemm_i8_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, GemmParams p, int use_tma_store) {
  using Cfg = PairCfg<EPI, OUT_DT, B_INT4>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * Cfg::A_BYTES;
  uint8_t* sBP = sB + STAGES * Cfg::B_BYTES;  // [STAGES][128 rows][64 B] packed (B_INT4)
  uint8_t* sC = sBP + STAGES * Cfg::BP_BYTES;  // [EPI_WARPS][EPI_STAGE_BYTES] (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;     // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* drain = tempty + 2;         // abort path: the MMA issuer's last commit
  uint64_t* conv = drain + 1;           // [STAGES] B_INT4, leader: both CTAs' halves unpacked
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(conv + (B_INT4 ? STAGES : 0));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      if constexpr (B_INT4) mbar_init(&conv[s], 2 * Cfg::UNPACK_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * EPI_WARPS);
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

  const int num_m = (p.M + 2 * GEMM_BM - 1) / (2 * GEMM_BM);
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (p.K + GEMM_BK - 1) / GEMM_BK;
  // split K / narrow last wave: see GemmParams
  const int num_units = SPLIT ? num_tiles * p.splits : full_or_narrow_units(p, num_tiles);
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  // Launched with PDL, everything above overlaps the previous kernel's tail;
  // no global memory is read or written before pdl_wait.  (An L2 prefetch of
  // the first tile's weight slabs here measured no gain.)
  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      ArmedLoads armed;  // both CTAs' loads complete on the leader's barriers
      bool ok = true;
      for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
        const int kb0 = SPLIT ? (u / num_tiles) * p.kb_split : 0;
        const int kb1 = SPLIT ? min(kb0 + p.kb_split, num_kb) : num_kb;
        int mb, n0, width = BN;
        if constexpr (SPLIT) {
          int nb;
          tile_coords(u % num_tiles, num_m, num_n, mb, nb);
          n0 = nb * BN;
        } else {
          width = unit_geometry<BN>(p, u, num_m, num_n, mb, n0);
        }
        const int arow = mb * 2 * GEMM_BM + (int)rank * GEMM_BM;
        // each CTA holds half of the unit's weight rows (a narrow unit's MMA
        // reads the first 64 of the 128 loaded)
        const int brow = n0 + (int)rank * (width / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          if (!(kb == p.stall_kb && u == cluster_id)) {
            if constexpr (B_INT4) {  // own barrier: this CTA's unpack warps wait on it
              mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::BP_BYTES);
              tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * GEMM_BK, arow);
              tma_load_2d(sBP + stage * Cfg::BP_BYTES, &tmB, &full[stage], kb * (GEMM_BK / 2), brow);
            } else {
              const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
              if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
              if (p.a_seg == 0) tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, fb, kb * GEMM_BK, arow);
              else tma_load_3d_pair(sA + stage * Cfg::A_BYTES, &tmA, fb, kb * GEMM_BK, arow % p.a_seg, arow / p.a_seg);
              tma_load_2d_pair(sB + stage * Cfg::B_BYTES, &tmB, fb, kb * GEMM_BK, brow);
            }
            armed.note(stage, phase);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // no load still writing shared memory at exit: the peer CTA cannot
      // pass the final cluster barrier before the leader has seen both CTAs'
      // loads land on its barriers (packed B: each CTA's own barriers)
      if (leader || B_INT4) armed.drain(full, STAGES);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      constexpr uint32_t idesc_full = umma_idesc_i8(2 * GEMM_BM, BN);
      constexpr uint32_t idesc_narrow = umma_idesc_i8(2 * GEMM_BM, BN / 2);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false, ok = true;
      for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
        const int kb0 = SPLIT ? (u / num_tiles) * p.kb_split : 0;
        const int kb1 = SPLIT ? min(kb0 + p.kb_split, num_kb) : num_kb;
        const uint32_t idesc = (!SPLIT && p.narrow_first > 0 && u >= p.narrow_first) ? idesc_narrow : idesc_full;
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(B_INT4 ? &conv[stage] : &full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = umma_desc_k_sw128(smem_u32(sA + stage * Cfg::A_BYTES));
          const uint64_t bdesc = umma_desc_k_sw128(smem_u32(sB + stage * Cfg::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 32; ++k)
            umma_i8_pair(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          issued = true;
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      if (*abort_flag && issued) {  // MMAs complete before TMEM is released
        umma_commit_pair(drain, 0x1);
        mbar_wait_drain(drain, 0);
      }
    }
  } else if (B_INT4 && warp >= 2 + EPI_WARPS) {
    // ---------------- int4 -> 16*int4 unpack of this CTA's 128 weight rows ----------------
    // (warp 10 + j: rows 64*j..; the MMA waits on the leader's conv barrier)
    const int part = warp - (2 + EPI_WARPS);
    const uint32_t conv_leader0 = mapa_shared(smem_u32(&conv[0]), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = cluster_id; ok && u < num_units; u += num_clusters) {
      const int kb0 = SPLIT ? (u / num_tiles) * p.kb_split : 0;
      const int kb1 = SPLIT ? min(kb0 + p.kb_split, num_kb) : num_kb;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&full[stage], phase, abort_flag)) { ok = false; break; }
        unpack_int4_rows64_warp(sBP + stage * Cfg::BP_BYTES, sB + stage * Cfg::B_BYTES, part, lane);
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
    // ---------------- epilogue (both CTAs) ----------------
    EpiSmem<BN>* es = reinterpret_cast<EpiSmem<BN>*>((reinterpret_cast<uintptr_t>(tmem_slot) + 16 + 15) & ~uintptr_t(15));
    const bool tma_st = Cfg::TMA_ST && use_tma_store;
    if (tma_st && lane == 0) tma_prefetch_desc(&tmC);
    epilogue_role<BN, EPI, OUT_DT, 2 * GEMM_BM, true, B_INT4 ? 4 : 0, SPLIT>(p, es, tfull, tempty, abort_flag, tmem_base, cluster_id,
                                                      num_clusters, num_tiles, num_m, num_n, (int)rank * GEMM_BM, warp,
                                                      lane, tma_st ? &tmC : nullptr,
                                                      sC + (warp - 2) * Cfg::EPI_BUFS * EPI_STAGE_BYTES);
  }

  tc_fence_before();
  cluster_sync();  // all MMAs done and all remote arrivals delivered
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace qlin
