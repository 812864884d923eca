// Node-side GEMMs of the fp16 engine on tcgen05 tensor cores:
//   C[M, N] = act(A[M, K] W^T + b),   A and W fp32, C fp32 or fp16
// (the encoder's node terms, its node FFN and W3, and the decoder's per-residue
// tables; M = residues).  Both operands are applied as an fp16 value plus an
// fp16 remainder, x = hi + lo with lo = fp16(x - hi), and the product is formed
// as three MMAs into one fp32 accumulator,
//   W_hi A_hi + W_hi A_lo + W_lo A_hi,
// which keeps about 22 significant bits of each operand (the dropped
// W_lo A_lo term is below 2^-22 of the product), i.e. close to the fp32 SIMT
// result it replaces at a fraction of the time.
//
// One CTA per (128-row tile, 128-column block): the weights are the A operand
// (M = 128 output features on TMEM lanes), the activation rows the B operand
// (N = 128 rows on TMEM columns).  K advances one 64-column atom at a time
// through a shared-memory stage: thread 0 loads the weight atoms (value and
// remainder images prepared at engine creation) by bulk copy, the 512 threads
// load the fp32 activation atom and split it into the value and remainder
// operand atoms, and thread 0 issues the three K = 64 products and commits
// them to the stage's mbarrier.  Two CTAs share an SM, so one CTA's loads and
// epilogue overlap the other's products.  The epilogue adds the bias, applies the activation
// (the reference's erf GELU) and stores rows feature-contiguous (a warp writes
// 32 consecutive columns of one row).  Every wait is bounded.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace hkb {
namespace {

using namespace tc;

// One stage (64 KiB) lets two CTAs share an SM, which measured faster than
// two stages (the activation load then overlaps the other CTA's products and
// epilogue instead of this CTA's own).
#ifndef HKB_GT_STAGES
#define HKB_GT_STAGES 1
#endif
constexpr int kGtThreads = 512;
constexpr int kGtStages = HKB_GT_STAGES;          // shared-memory stages
constexpr uint32_t kGtAtom = 128 * 128;           // 128 rows x 64 fp16 (SW128)
constexpr uint32_t kGtStage = 4 * kGtAtom;        // W hi, W lo, A hi, A lo
constexpr uint32_t kGtSmem = kGtStages * kGtStage + 1024;

__device__ __forceinline__ uint32_t idesc_h16(int M, int N) {
  return idesc_bf16(M, N) & ~((7u << 7) | (7u << 10));
}

// K = 64 product of one 128-row A atom and one 128-row B atom (both SW128
// K-major): four K = 16 MMAs; accumulates when `acc` is set.
__device__ __forceinline__ void mma_k64(uint32_t d_tmem, uint32_t a_smem, uint32_t b_smem,
                                        uint32_t idesc, bool acc) {
  const uint64_t da = sw128_desc(a_smem), db = sw128_desc(b_smem);
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    mma_bf16(d_tmem, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc,
             (acc || kk > 0) ? 1u : 0u);
}

// fp16 pair of (a, b) (lo = false) or of their remainders a - fp16(a),
// b - fp16(b) (exact in fp32).
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int ACT, bool OUT16>
__global__ void __launch_bounds__(kGtThreads, 3 - kGtStages) gemm_tc3_kernel(
    int64_t M, int K, const float* __restrict__ A, int lda,
    const unsigned char* __restrict__ Whi, const unsigned char* __restrict__ Wlo,
    const float* __restrict__ bias, void* __restrict__ C, int ldc, unsigned int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t bar_w[2], bar_mma[2];
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cgrp = warp >> 2;   // TMEM lane quadrant, 32-row column group
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int64_t m0 = (int64_t)blockIdx.x * 128;
  const int nb = blockIdx.y;
  const int nk = K / 64;

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_w[s], 1);
      mbar_init(&bar_mma[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  const unsigned char* wh = Whi + (size_t)nb * nk * kGtAtom;
  const unsigned char* wl = Wlo + (size_t)nb * nk * kGtAtom;
  const uint32_t idesc = idesc_h16(128, 128);
  uint32_t ph_w[2] = {0u, 0u}, ph_m[2] = {0u, 0u};
  bool ok = true;

  // this thread's share of an activation atom: row tid / 4, 16 columns
  const int ar = tid >> 2, ac = (tid & 3) * 16;
  const int64_t arow = m0 + ar;
  for (int ka = 0; ka < nk; ++ka) {
    const int s = ka % kGtStages;
    unsigned char* st = sm + s * kGtStage;
    if (ka >= kGtStages) {   // stage s was last read by the products of atom ka - kGtStages
      if (!mbar_wait(&bar_mma[s], ph_m[s], err)) ok = false;
      ph_m[s] ^= 1;
      tc_fence_after();
    }
    if (tid == 0) {
      mbar_arrive_expect_tx(&bar_w[s], 2 * kGtAtom);
      bulk_g2s(st, wh + (size_t)ka * kGtAtom, kGtAtom, &bar_w[s]);
      bulk_g2s(st + kGtAtom, wl + (size_t)ka * kGtAtom, kGtAtom, &bar_w[s]);
    }
    {
      float v[16];
      if (arow < M) {
        const float4* src = reinterpret_cast<const float4*>(A + arow * lda + ka * 64 + ac);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 x = src[q];
          v[4 * q] = x.x;
          v[4 * q + 1] = x.y;
          v[4 * q + 2] = x.z;
          v[4 * q + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        uint32_t h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) split2(v[8 * u + 2 * i], v[8 * u + 2 * i + 1], h[i], l[i]);
        const uint32_t off = sw128_offset(ar, ac + 8 * u, 128);
        *reinterpret_cast<uint4*>(st + 2 * kGtAtom + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(st + 3 * kGtAtom + off) = make_uint4(l[0], l[1], l[2], l[3]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      if (!mbar_wait(&bar_w[s], ph_w[s], err)) ok = false;
      tc_fence_after();
      const uint32_t swh = smem_u32(st), swl = smem_u32(st + kGtAtom);
      const uint32_t sah = smem_u32(st + 2 * kGtAtom), sal = smem_u32(st + 3 * kGtAtom);
      if (ok) {
        mma_k64(tm, swh, sah, idesc, ka > 0);
        mma_k64(tm, swh, sal, idesc, true);
        mma_k64(tm, swl, sah, idesc, true);
      }
      mma_commit(&bar_mma[s]);
    }
    ph_w[s] ^= 1;
  }
  // the last commit covers every product of thread 0
  {
    const int s = (nk - 1) % kGtStages;
    if (!mbar_wait(&bar_mma[s], ph_m[s], err)) ok = false;
    tc_fence_after();
  }
  // epilogue: TMEM lane = output feature, columns = rows of the tile
  const int f = quad * 32 + lane;
  const int n = nb * 128 + f;
  const float b = bias ? bias[n] : 0.0f;
  {
    float v[32];
    tmem_ld32(tm + lane_base + (uint32_t)(cgrp * 32), v);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int64_t row = m0 + cgrp * 32 + i;
      if (row < M) {
        float y = v[i] + b;
        if (ACT == 1) y = gelu_as(y);
        if constexpr (OUT16)
          reinterpret_cast<__half*>(C)[row * ldc + n] = __float2half_rn(y);
        else
          reinterpret_cast<float*>(C)[row * ldc + n] = y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 128);
}

}  // namespace

void gemm_tc3(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
              const unsigned char* Whi, const unsigned char* Wlo, const float* bias, int act,
              void* C, int ldc, bool out_f16, unsigned int* err) {
  if (M <= 0) return;
  ensure_dynamic_smem((const void*)gemm_tc3_kernel<0, false>, (int)kGtSmem);
  ensure_dynamic_smem((const void*)gemm_tc3_kernel<1, false>, (int)kGtSmem);
  ensure_dynamic_smem((const void*)gemm_tc3_kernel<0, true>, (int)kGtSmem);
  const dim3 grid((unsigned)((M + 127) / 128), (unsigned)(N / 128));
  if (out_f16)
    gemm_tc3_kernel<0, true><<<grid, kGtThreads, kGtSmem, st>>>(M, K, A, lda, Whi, Wlo, bias, C,
                                                               ldc, err);
  else if (act == 1)
    gemm_tc3_kernel<1, false><<<grid, kGtThreads, kGtSmem, st>>>(M, K, A, lda, Whi, Wlo, bias, C,
                                                                ldc, err);
  else
    gemm_tc3_kernel<0, false><<<grid, kGtThreads, kGtSmem, st>>>(M, K, A, lda, Whi, Wlo, bias, C,
                                                                ldc, err);
}

}  // namespace hkb
