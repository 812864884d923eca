// Hand-written sm_100a building blocks: mbarriers with bounded waits, 1-D
// bulk copies (TMA engine, no tensor map), tensor memory (TMEM) allocation and
// loads, and tcgen05.mma with shared-memory matrix descriptors.
//
// Operand layout: every MMA operand is a K-major tile stored with the 128-byte
// swizzle.  For a tile of R rows (R a multiple of 8) and K bf16 columns, the
// columns are cut into 64-element "atoms"; atom a occupies R*128 bytes, rows
// are 128 bytes apart inside 1024-byte groups of 8 rows, and the 16-byte chunk
// c of row r sits at chunk position c ^ (r % 8).  Tile bases are 1024-byte
// aligned.  sw128_offset() gives the byte offset of element (r, k).
//
// Descriptor encodings follow the PTX ISA tables for tcgen05 (matrix
// descriptor: start >> 4 at bits 0-13, leading offset >> 4 at 16-29, stride
// offset >> 4 at 32-45, version 1 at 46, swizzle mode at 61-63; instruction
// descriptor for kind::f16: D format at 4-5, A/B formats at 7-9 / 10-12,
// major bits 15/16, N >> 3 at 17-22, M >> 4 at 24-28).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace hkb {
namespace tc {

__host__ __device__ constexpr uint32_t sw128_offset(int r, int k, int rows) {
  return (uint32_t)((k >> 6) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    ((((k & 63) >> 3) ^ (r & 7)) << 4) + (k & 7) * 2);
}

// Instruction descriptor: D f32, A and B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Matrix descriptor of a SW128 K-major tile starting at shared address `a`.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t a) {
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// ---- mbarrier -------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
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

// Waits for phase `parity` of `bar` to complete, for at most ~1 s of SM
// clock.  On timeout it records kErrTimeout and returns false; callers then
// skip work and finish, so a kernel never hangs on a barrier.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (2LL << 30)) {
      if (err) atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// Like mbar_wait, but also gives up (without recording a timeout) as soon as
// another thread of the CTA has raised `*abort`.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity,
                                                    unsigned int* err, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (clock64() - t0 > (2LL << 30)) {
      if (err) atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier over `count` threads (a multiple of 32); id 0 is __syncthreads.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- bulk copy global -> shared (completes bytes on an mbarrier) ----------
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- tiled TMA load (tensor map, no multicast) -------------------------------
// Copies the box at element coordinates (x, y) of the 2-D tensor `map` (x the
// innermost coordinate) into shared memory at `dst` and completes its bytes on
// `bar`.  Boxes with the 128-byte swizzle need a 1024-byte aligned `dst`, and
// x * element size must be a multiple of 16 bytes; rows past the tensor's
// extent read as zero.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of a contiguous global range (both the address and the size a
// multiple of 16 bytes); nothing waits on it.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte global loads that do not allocate in L1, for rows read once: they
// would otherwise evict the small per-layer vectors that L1 keeps.  The .nc
// form is for data that no thread writes during the kernel; the plain form
// (ordered like any other memory access) for rows this kernel wrote.
__device__ __forceinline__ uint4 ld_nc_noalloc_v4(const void* p) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_noalloc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Generic-proxy shared-memory writes become visible to the async proxy
// (tensor cores, bulk copies).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tensor memory ----------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, one instruction (K = 16 for bf16).
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every previously issued tcgen05.mma of this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// K = 128 product of one 128-row A tile and an N-row B tile (both SW128
// K-major, 2 atoms along K), accumulating into D when `acc` is set.  The
// descriptor's start-address field (address >> 4, 14 bits) is linear in the
// address and shared memory lies below 256 KB, so step kk's descriptors are
// the tile's base descriptors plus (offset >> 4): no field can carry.
__device__ __forceinline__ void mma_k128(uint32_t d_tmem, uint32_t a_smem, uint32_t b_smem,
                                         int n_rows, uint32_t idesc, bool acc) {
  const uint64_t da = sw128_desc(a_smem), db = sw128_desc(b_smem);
  const uint64_t b_atom = (uint64_t)((uint32_t)n_rows * 128u >> 4);
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const uint64_t off = (uint64_t)((kk & 3) * 2);   // 32 bytes >> 4
    mma_bf16(d_tmem, da + (uint64_t)(kk >> 2) * (128u * 128u >> 4) + off,
             db + (uint64_t)(kk >> 2) * b_atom + off, idesc, (acc || kk > 0) ? 1u : 0u);
  }
}

// 32 lanes x 16 (or 32) consecutive 32-bit columns per warp, followed by
// tcgen05.wait::ld inside the same asm statement so no use of the outputs can
// be scheduled before the load has landed.  Lane i of the warp reads TMEM lane
// 32 * (warp % 4) + i; the caller folds that lane base into taddr.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 48 consecutive columns (an x32 and an x16 load) with one wait.
__device__ __forceinline__ void tmem_ld48(uint32_t taddr, float (&v)[48]) {
  uint32_t r[48];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%48];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47}, [%49];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
        "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]),
        "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47])
      : "r"(taddr), "r"(taddr + 32u)
      : "memory");
#pragma unroll
  for (int i = 0; i < 48; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc
}  // namespace hkb
