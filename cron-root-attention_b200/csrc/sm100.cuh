// sm100.cuh -- thin inline-PTX layer over the Blackwell (sm_100a) primitives the
// attention kernels use: mbarriers, TMA tile loads, TMEM allocation, tcgen05
// MMA / commit / load / store, and the shared-memory matrix descriptors.
//
// Conventions used by every kernel in this library:
//  * A [rows x D] bf16/f16 tile in shared memory is stored as D/64 "chunks",
//    each chunk [rows x 128 B] in the 128-byte swizzled layout TMA writes with
//    CU_TENSOR_MAP_SWIZZLE_128B (16-byte unit u of row r sits at u ^ (r & 7)).
//    Chunk c holds columns [64c, 64c+64) and starts at c * rows * 128 bytes.
//    Every chunk base is 1024-byte aligned.
//  * That layout is the UMMA "K-major, SWIZZLE_128B" canonical layout when the
//    64-column direction is the contraction (K) direction (SBO = 1024 B between
//    8-row groups), and the "MN-major, SWIZZLE_128B" layout when the 64-column
//    direction is the M/N direction (LBO = chunk stride, SBO = 1024 B).
//  * Every wait is bounded (wall-clock limit from %globaltimer).  A wait that
//    runs out records an error code in global memory and sets a CTA-wide abort
//    flag; all later waits return at once, so the CTA drains and exits
//    normally (TMEM is always freed).  Nothing here traps.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace cra {

// ---------------------------------------------------------------------------
// error codes written by device code into the caller's error word
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,
};

#ifndef CRA_WAIT_LIMIT_NS
#define CRA_WAIT_LIMIT_NS 500000000ull  // 0.5 s: far above any legitimate wait
#endif
// Limit of the drain waits on abort paths (copies and MMAs already in flight
// always complete; this only bounds the spin).  Kept separate so that a build
// with a tiny CRA_WAIT_LIMIT_NS still lets in-flight work land.
#ifndef CRA_DRAIN_LIMIT_NS
#define CRA_DRAIN_LIMIT_NS 500000000ull
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// CTA-wide abort state shared by all waits of one CTA.
struct Abort {
  volatile int* flag;  // shared memory
  int* err;            // global error word (may be null)
};

// Bounded wait on phase `parity` of barrier `bar`.  Returns false if the CTA
// is aborting (this wait timed out, or another one did).
// try_waits between two reads of the clock and of the abort flag
#ifndef CRA_WAIT_POLLS
#define CRA_WAIT_POLLS 16
#endif
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < CRA_WAIT_POLLS; ++i)
      if (mbar_try(bar, parity)) return true;
    if (*ab.flag) return false;
    if (globaltimer() - t0 > CRA_WAIT_LIMIT_NS) {
      *ab.flag = 1;
      if (ab.err) atomicExch(ab.err, kDevWaitTimeout);
      return false;
    }
  }
}

// Bounded wait by a whole warp with a warp-uniform result (every lane polls;
// each lane leaves on completion, on the CTA abort flag or on its own time
// limit, so the vote always completes).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, ab));
}

// ---------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 4-D tiled load (coordinates innermost first) into CTA shared memory,
// completing `bytes` on barrier `bar`.  No multicast.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// L2 prefetch of one 4-D tile (no shared memory written, nothing to wait for).
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* m, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing `bytes` on barrier `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// ---------------------------------------------------------------------------
// TMEM + tcgen05
// ---------------------------------------------------------------------------
// Warp-collective: allocates `ncols` TMEM columns, address written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (a tcgen05.mma operand, a TMA store).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100
// descriptor version 1.  Addresses / offsets in bytes.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//  bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 f16, 1 bf16),
//  15 A major (0 K, 1 MN), 16 B major, 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// MMA issue.  The whole warp executes these calls with warp-uniform operands
// and one elected lane (always the same: the lowest) issues.  Issuing from a
// converged warp keeps the descriptors on the uniform datapath; a lone thread
// in a divergent branch sustains only about one MMA per ~90 cycles (measured
// on B200), which caps M128 x N64 x K16 MMAs at about a third of the
// tensor-core rate.  MMAs issued this way execute in issue order.
//
// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss_w(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Copies a 128-row x 32-byte matrix (one K-step of 16 16-bit elements of a
// K-major operand, described like an MMA operand) from shared memory to TMEM:
// row i -> lane i, 8 consecutive columns, the layout a TS-form MMA reads its A
// operand in.  Executes in order before later MMAs of the issuing thread.
__device__ __forceinline__ void tmem_cp_128x256b_w(uint32_t taddr, uint64_t s) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.cp.cta_group::1.128x256b [%0], %1;\n\t}" ::"r"(taddr), "l"(s)
      : "memory");
}
// Arrive on `bar` once every MMA the elected lane issued so far has completed
// (a commit covers all earlier MMAs of the thread, not just the latest).
__device__ __forceinline__ void mma_commit_w(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit: each thread gets 32 consecutive columns of
// its own lane (row).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%"
      "20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 columns store (16 x 32-bit per thread).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed two-lane fp32 arithmetic (one instruction for two values).
// a = a * b + c on both lanes
__device__ __forceinline__ void ffma2(float& a0, float& a1, float b, float c) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %2};\n\tmov.b64 z, {%3, %3};\n\t"
      "fma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b), "f"(c));
}
// a += b on both lanes
__device__ __forceinline__ void fadd2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// Two-lane vector forms on float2 (one f32x2 instruction each).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {  // a * b + c
  float2 d;
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%6, %7};\n\t"
      "fma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "mul.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Hardware base-2 exponential (MUFU.EX2), flush-to-zero.  ex2(-inf) = +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32-byte global store (one full sector per thread); 32-byte aligned address.
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t (&w)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Stores 8 words at p: one 32-byte store when v8 (p 32-byte aligned), else
// two 16-byte stores (p 16-byte aligned).
__device__ __forceinline__ void st_global_8w(void* p, const uint32_t (&w)[8], bool v8) {
  if (v8) {
    st_global_v8(p, w);
  } else {
    uint4* q = reinterpret_cast<uint4*>(p);
    q[0] = make_uint4(w[0], w[1], w[2], w[3]);
    q[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Bounded spin used only on abort paths (no abort flag to consult).
__device__ __forceinline__ void mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try(bar, parity) && globaltimer() - t0 < CRA_DRAIN_LIMIT_NS) {
  }
}

// ---------------------------------------------------------------------------
// element type helpers
// ---------------------------------------------------------------------------
template <bool BF16>
struct Elt;
template <>
struct Elt<true> {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
  }
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elt<false> {
  using T = __half;
  using T2 = __half2;
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t u) { return __half22float2(*reinterpret_cast<__half2*>(&u)); }
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
};

}  // namespace cra
