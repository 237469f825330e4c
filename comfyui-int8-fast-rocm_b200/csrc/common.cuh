// Shared device helpers for the sm_100a quantized-linear kernels: dtype
// conversion with explicit IEEE rounding, in-register Hadamard stages, and
// mbarrier / TMA / tcgen05 PTX wrappers.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qlin {

enum : int { DT_BF16 = 0, DT_F16 = 1, DT_F32 = 2 };
enum : int { ROT_NONE = 0, ROT_REGULAR = 1, ROT_SYLVESTER = 2 };

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <int DT> struct Elem;
template <> struct Elem<DT_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Elem<DT_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Elem<DT_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f(T v) { return v; }
  static __device__ __forceinline__ T from_f(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};

// Load 16 consecutive elements (16-byte aligned) as float.
template <int DT>
__device__ __forceinline__ void load16(const typename Elem<DT>::T* p, float (&v)[16]) {
  if constexpr (DT == DT_F32) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float4 t = __ldg(q + i);
      v[4 * i + 0] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
    }
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      uint4 t = __ldg(q + i);
      uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (DT == DT_BF16) {
          v[8 * i + 2 * j + 0] = __uint_as_float(w[j] << 16);
          v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
        } else {
          __half2 h = *reinterpret_cast<__half2*>(&w[j]);
          float2 f = __half22float2(h);
          v[8 * i + 2 * j + 0] = f.x;
          v[8 * i + 2 * j + 1] = f.y;
        }
      }
    }
  }
}

// Store 16 floats (already representable in DT) as DT, 16-byte aligned.
template <int DT>
__device__ __forceinline__ void store16(typename Elem<DT>::T* p, const float (&v)[16]) {
  if constexpr (DT == DT_F32) {
    float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else {
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if constexpr (DT == DT_BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
    }
    uint4* q = reinterpret_cast<uint4*>(p);
    q[0] = make_uint4(w[0], w[1], w[2], w[3]);
    q[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

// Integer value of round-half-even(v) for |v| < 2^22: adding 1.5*2^23 moves
// the integer part into the low mantissa bits with one full-rate float add.
__device__ __forceinline__ int rint_to_int(float v) {
  return __float_as_int(__fadd_rn(v, 12582912.0f)) - 0x4B400000;
}

// ---------------------------------------------------------------------------
// In-register Hadamard stages (fixed float32 evaluation order; the oracle
// evaluates the identical expressions)
// ---------------------------------------------------------------------------
// Regular H4 (convrot.py:40-43): every column sums the 4 inputs and flips the
// sign of exactly one (anti-diagonal), so y_k = S - 2*a_{3-k}.
__device__ __forceinline__ void h4_regular(float& a0, float& a1, float& a2, float& a3) {
  // fma(-2, a, s) == RN(s - 2a): 2a is exact, so this is the same single
  // rounding as a subtraction of the doubled value.
  const float s = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
  const float y0 = __fmaf_rn(-2.0f, a3, s);
  const float y1 = __fmaf_rn(-2.0f, a2, s);
  const float y2 = __fmaf_rn(-2.0f, a1, s);
  const float y3 = __fmaf_rn(-2.0f, a0, s);
  a0 = y0; a1 = y1; a2 = y2; a3 = y3;
}
__device__ __forceinline__ void h2_sylvester(float& a0, float& a1) {
  const float y0 = __fadd_rn(a0, a1);
  const float y1 = __fsub_rn(a0, a1);
  a0 = y0; a1 = y1;
}

// Transform over the low log2(N) index bits of v[N] (N in {2,4,8,16}),
// digit by digit from the least significant one.
template <int KIND, int N>
__device__ __forceinline__ void xform_regs(float* v) {
  if constexpr (KIND == ROT_REGULAR) {
    static_assert(N == 4 || N == 16, "regular Hadamard digits are base 4");
#pragma unroll
    for (int stride = 1; stride < N; stride *= 4) {
#pragma unroll
      for (int base = 0; base < N; base += 4 * stride) {
#pragma unroll
        for (int o = 0; o < stride; ++o) {
          h4_regular(v[base + o], v[base + o + stride], v[base + o + 2 * stride], v[base + o + 3 * stride]);
        }
      }
    }
  } else if constexpr (KIND == ROT_SYLVESTER) {
#pragma unroll
    for (int stride = 1; stride < N; stride *= 2) {
#pragma unroll
      for (int base = 0; base < N; base += 2 * stride) {
#pragma unroll
        for (int o = 0; o < stride; ++o) h2_sylvester(v[base + o], v[base + o + stride]);
      }
    }
  }
}

// Packed float32x2 arithmetic (sm_100): two IEEE float32 operations per
// instruction on a register pair, each rounded to nearest even.
// Caution: a packed multiply whose only use is a following packed add has
// been fused into one FMA by the assembler (even with -fmad=false); code that
// needs those two roundings must not write that pair (rowquant_pair_kernel
// adds through an FMA with a run-time 1.0 instead).
__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 f2_add(float2 a, float2 b) { return __fadd2_rn(a, b); }
// a * b + c with one rounding per component.
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ---------------------------------------------------------------------------
// PTX wrappers: shared-memory addresses, mbarriers, TMA, tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled TMA store shared -> global (bulk-group completion).  Elements of
// the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// 3-D form of tma_store_2d.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the shared-memory sources of this thread's committed bulk stores may be reused
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// all but the most recent of this thread's committed bulk stores have read their shared-memory source
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// this thread's committed bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-D bulk copy global -> this CTA's shared memory (no multicast), counted on
// an mbarrier; addresses 16-byte aligned, size a multiple of 16 bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (a hint; 16-byte aligned,
// size a multiple of 16 bytes, inside one allocation).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// tcgen05 --------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on an mbarrier when all prior tcgen05.mma of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}


// ---- thread-block clusters and the CTA-pair (cta_group::2) tcgen05 forms ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Programmatic dependent launch (launch_pdl on the host): pdl_wait returns
// once the previous kernel of the stream has completed and its memory
// operations are visible (immediately for a plain launch); after
// pdl_launch_dependents in every CTA, the next kernel of the stream, if
// launched with PDL, may be scheduled and start its own set-up.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Remote mbarrier arrival with the default semantics (release, CTA scope),
// as CUTLASS's cluster barriers arrive: a cluster-scope release waits for
// the memory system (about 1200 cycles per arrival, measured on B200).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of the CTA pair (here: the leader's), no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint32_t mbar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(mbar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
// 3-D form of tma_load_2d_pair (segmented rows: {column, row in segment,
// segment}).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* tmap, uint32_t mbar_cluster_addr, int x, int y,
                                                 int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(mbar_cluster_addr), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[smem of both] . B[smem of both]^T, M = 256.
__device__ __forceinline__ void umma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the mbarrier at the same offset in every CTA of `mask` when all
// prior pair MMAs of this thread complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld tied to the registers of one earlier tmem_ld_32x32b_x32:
// they are in-out operands of the wait, so no use of them can be scheduled
// before it (the load writes them asynchronously).
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzle: rows of 128 bytes, 8-row core groups 1024 bytes
// apart (SBO), LBO unused (1), descriptor version 1, layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;            // LBO (ignored for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // SBO
  d |= static_cast<uint64_t>(1) << 46;            // version
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::i8, signed A and B, S32 accumulator,
// both operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
  return (2u << 4)            // D format S32
         | (1u << 7)          // A signed int8
         | (1u << 10)         // B signed int8
         | (0u << 15)         // A K-major
         | (0u << 16)         // B K-major
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// SiTU gated activation (int8_fused_kernel.py:389-421), float32 math with
// every step an explicit round-to-nearest operation, so the standalone
// kernel and the quantiser prologue that share it produce identical values.
// tanh without overflow: (1 - e^-2|x|) / (1 + e^-2|x|) with the sign
// restored, and the odd Taylor polynomial x(1 - x^2(1/3 - 2x^2/15)) below
// |x| = 0.02 where the quotient cancels (int8_fused_kernel.py:390-399).
__device__ __forceinline__ float situ_tanh(float x) {
  const float ax = fabsf(x);
  const float t = expf(__fmul_rn(-2.0f, ax));
  float big = __fdiv_rn(__fsub_rn(1.0f, t), __fadd_rn(1.0f, t));
  big = x < 0.0f ? -big : big;
  const float x2 = __fmul_rn(x, x);
  const float inner = __fsub_rn(1.0f / 3.0f, __fmul_rn(x2, 2.0f / 15.0f));
  const float small = __fmul_rn(x, __fsub_rn(1.0f, __fmul_rn(x2, inner)));
  return ax < 0.02f ? small : big;
}
// out = 4 tanh(g/4) * sigmoid(g) * 25 tanh(h/25)  (int8_fused_kernel.py:403-421)
__device__ __forceinline__ float situ_f(float h, float g) {
  const float gate_cap = __fmul_rn(4.0f, situ_tanh(__fmul_rn(g, 0.25f)));
  const float hidden_cap = __fmul_rn(25.0f, situ_tanh(__fdiv_rn(h, 25.0f)));
  return __fmul_rn(__fdiv_rn(gate_cap, __fadd_rn(1.0f, expf(-g))), hidden_cap);
}

}  // namespace qlin
