// Persistent tcgen05 GEMM for the tensor-core modes:
//   C[M, N] = act(A[M, K] . W[N, K]^T + bias[N])
// A is fp32 or fp16 in global memory (row-major, leading dimension lda); each
// 128-row tile is converted to fp16 and stored in the SW128 K-major layout, K
// in chunks of 128 (two 64-column atoms), double-buffered so the next chunk
// loads while the tensor cores consume the current one.  W is a pre-swizzled
// fp16 image ([K/64 atoms][N rows x 64]) loaded once per CTA by bulk copies and
// kept resident.  The accumulator D[128 rows, N] lives in TMEM (lanes = rows);
// the epilogue adds the bias, applies GELU if asked (exact erf form: these
// GEMMs are memory-bound, and the encoder's accuracy depends on it), and
// writes fp32 or fp16.
// N is a multiple of 128 up to 512 (MMAs of N <= 256); K up to 512.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace hkb {
namespace {

using namespace tc;

constexpr int kGemmThreads = 256;
constexpr uint32_t kAChunkBytes = 128 * 128 * 2;   // 32 KiB per K chunk

template <bool AF16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    linear_tc_kernel(const __grid_constant__ LinearTcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int Kp = (p.K + 63) & ~63;                       // padded K (atoms)
  const uint32_t w_bytes = (uint32_t)p.N * (uint32_t)Kp * 2u;
  unsigned char* sW = sm;
  unsigned char* sA = sm + ((w_bytes + 1023u) & ~1023u); // 2 x 32 KiB
  __shared__ uint64_t bar_w, bar_a[2], bar_d;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;                      // TMEM lane / tile row
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  // K chunk: 128 columns (two atoms).
  const int kchunk = 128;
  const int nchunks = (Kp + kchunk - 1) / kchunk;
  const uint32_t ncols = p.N <= 256 ? 256u : 512u;

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_a[0], 1);
    mbar_init(&bar_a[1], 1);
    mbar_init(&bar_d, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    // resident weight image, bulk copies of at most 64 KiB
    mbar_arrive_expect_tx(&bar_w, w_bytes);
    for (uint32_t o = 0; o < w_bytes; o += 65536u) {
      const uint32_t n = (w_bytes - o) < 65536u ? (w_bytes - o) : 65536u;
      bulk_g2s(sW + o, p.W + o, n, &bar_w);
    }
  }
  uint32_t ph_a = 0;     // bit b: parity of A buffer b's next barrier phase
  uint32_t ph_d = 0;
  bool w_ready = false;
  // bit b: an MMA group committed on A buffer b is still owed its wait (same on
  // all threads; bit masks rather than arrays indexed by b, which would sit in
  // local memory)
  uint32_t owed = 0;

  const int64_t tiles = (p.M + 127) / 128;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    if (__syncthreads_or(abort_flag)) break;
    const int64_t m0 = t * 128;
    for (int c = 0; c < nchunks; ++c) {
      const int b = c & 1;
      // the MMAs that last read buffer b must be done before it is refilled
      if ((owed >> b) & 1u) {
        if (!mbar_wait(&bar_a[b], (ph_a >> b) & 1u, p.err)) abort_flag = 1;
        ph_a ^= 1u << b;
        owed &= ~(1u << b);
      }
      unsigned char* dst = sA + b * kAChunkBytes;
      const int k0 = c * kchunk;
      const int kw = (Kp - k0) < kchunk ? (Kp - k0) : kchunk;   // 64 or 128 columns
      // each warp fills rows; a lane converts 4 consecutive columns
      for (int r = warp; r < 128; r += kGemmThreads / 32) {
        const int64_t gm = m0 + r;
        for (int cc = lane * 4; cc < kw; cc += 128) {
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          const int gk = k0 + cc;
          if (gm < p.M) {
            if (AF16) {
              const __half* a = static_cast<const __half*>(p.A) + gm * p.lda + gk;
#pragma unroll
              for (int u = 0; u < 4; ++u) v[u] = (gk + u < p.K) ? __half2float(a[u]) : 0.f;
            } else {
              const float* a = static_cast<const float*>(p.A) + gm * p.lda + gk;
              if (gk + 3 < p.K && (p.lda & 3) == 0) {
                const float4 q = *reinterpret_cast<const float4*>(a);
                v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
              } else {
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = (gk + u < p.K) ? a[u] : 0.f;
              }
            }
          }
          const __half2 h0 = __floats2half2_rn(v[0], v[1]);
          const __half2 h1 = __floats2half2_rn(v[2], v[3]);
          uint2 pk;
          pk.x = *reinterpret_cast<const uint32_t*>(&h0);
          pk.y = *reinterpret_cast<const uint32_t*>(&h1);
          *reinterpret_cast<uint2*>(dst + sw128_offset(r, cc, 128)) = pk;

        }
      }
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        if (!w_ready) {
          if (!mbar_wait(&bar_w, 0, p.err)) abort_flag = 1;
          w_ready = true;
        }
        tc_fence_after();
        if (!abort_flag) {
          const int ksteps = kw / 16;
          for (int nb = 0; nb * 256 < p.N; ++nb) {
            const int nn = (p.N - nb * 256) < 256 ? (p.N - nb * 256) : 256;
            const uint32_t idesc = (idesc_bf16(128, nn) & ~((7u << 7) | (7u << 10)));  // fp16
            for (int kk = 0; kk < ksteps; ++kk) {
              const int atom = (k0 >> 6) + (kk >> 2);
              const uint32_t a = smem_u32(dst) + (uint32_t)(kk >> 2) * 128u * 128u + (kk & 3) * 32u;
              const uint32_t w = smem_u32(sW) + (uint32_t)atom * (uint32_t)p.N * 128u +
                                 (uint32_t)nb * 256u * 128u + (kk & 3) * 32u;
              mma_bf16(tm + nb * 256, sw128_desc(a), sw128_desc(w), idesc,
                       (c > 0 || kk > 0) ? 1u : 0u);
            }
          }
        }
        mma_commit(&bar_a[b]);
        if (c == nchunks - 1) mma_commit(&bar_d);
      }
      owed |= 1u << b;
    }
    // epilogue: wait for the accumulator, then rows out
    if (!mbar_wait(&bar_d, ph_d, p.err)) abort_flag = 1;
    ph_d ^= 1;
    tc_fence_after();
    const int64_t gm = m0 + row;
    const int ncol_half = p.N / 2;                 // warpgroup `half` writes its half
    for (int c0 = half * ncol_half; c0 < (half + 1) * ncol_half; c0 += 16) {
      float v[16];
      tmem_ld16(tm + lane_base + (uint32_t)c0, v);
      if (gm < p.M) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x = v[i] + (p.bias ? p.bias[c0 + i] : 0.0f);
          if (p.act == 1) x = 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
          v[i] = x;
        }
        if (p.out_f16) {
          __half* o = static_cast<__half*>(p.C) + gm * p.ldc + c0;
#pragma unroll
          for (int i = 0; i < 16; i += 8) {
            uint4 q;
            const __half2 a0 = __floats2half2_rn(v[i], v[i + 1]);
            const __half2 a1 = __floats2half2_rn(v[i + 2], v[i + 3]);
            const __half2 a2 = __floats2half2_rn(v[i + 4], v[i + 5]);
            const __half2 a3 = __floats2half2_rn(v[i + 6], v[i + 7]);
            q.x = *reinterpret_cast<const uint32_t*>(&a0);
            q.y = *reinterpret_cast<const uint32_t*>(&a1);
            q.z = *reinterpret_cast<const uint32_t*>(&a2);
            q.w = *reinterpret_cast<const uint32_t*>(&a3);
            *reinterpret_cast<uint4*>(o + i) = q;
          }
        } else {
          float* o = static_cast<float*>(p.C) + gm * p.ldc + c0;
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  // drain the A-buffer barriers still owed a wait, then the weight load
  for (int b = 0; b < 2; ++b)
    if ((owed >> b) & 1u) {
      mbar_wait(&bar_a[b], (ph_a >> b) & 1u, p.err);
      ph_a ^= 1u << b;
    }
  if (tid == 0 && !w_ready) mbar_wait(&bar_w, 0, p.err);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, ncols);
}

}  // namespace

size_t linear_tc_smem_bytes(int N, int K) {
  const size_t Kp = (size_t)((K + 63) & ~63);
  return (((size_t)N * Kp * 2 + 1023) & ~(size_t)1023) + 2 * kAChunkBytes + 1024;
}

void launch_linear_tc(cudaStream_t st, const LinearTcArgs& p, int num_sms) {
  if (p.M <= 0) return;
  const size_t smem = linear_tc_smem_bytes(p.N, p.K);
  // Largest request: N = 512, K = 128 or N = 128, K = 512 (193 KiB); the
  // opt-in limit also has to cover the kernel's static shared memory.
  static bool attr_set = false;
  if (!attr_set) {
    const int limit = (int)linear_tc_smem_bytes(512, 128);
    cudaFuncSetAttribute(linear_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         limit);
    cudaFuncSetAttribute(linear_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         limit);
    attr_set = true;
  }
  const int64_t tiles = (p.M + 127) / 128;
  const unsigned grid = (unsigned)(tiles < num_sms ? tiles : num_sms);
  if (p.a_f16)
    linear_tc_kernel<true><<<grid, kGemmThreads, smem, st>>>(p);
  else
    linear_tc_kernel<false><<<grid, kGemmThreads, smem, st>>>(p);
}

}  // namespace hkb
