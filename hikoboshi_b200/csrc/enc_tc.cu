// Fused tcgen05 encoder-layer kernels for the tensor-core modes.  h_E is kept
// in HBM as fp16 [R*48, 128] (slot s = residue * 48 + k) plus an fp16
// remainder array of the same shape (h_E = hi + lo, about 22 significant
// bits); MMAs read hi, the residual stream reads both.  Every edge-wise chain
// of an encoder layer runs in one pass over h_E, so no [R*48, 128]
// intermediate ever goes to HBM.  Weights are applied as fp16 value plus
// fp16 remainder (two MMAs into one fp32 accumulator):
//
//   enc_node_tc  (proteinmpnn_encoder_scalar.cpp:169-243)
//     D1 = W1b h_E                        M = 128 features, N = 192 slots
//     G  = GELU(D1 + [W1a h_i + b1] + W1c h_j)  (node terms gathered per slot)
//     D2 = W2 G
//     S_i = sum_k m_i m_j GELU(D2 + b2),  cnt_i = sum_k m_i m_j
//   Weights are the A operand and the 4 residues' 192 slots the B operand, so
//   a residue's 48 slots are 48 TMEM columns of one thread: the neighbour sum
//   is a thread-local loop in a fixed order (deterministic, no atomics).
//
//   enc_edge_tc  (proteinmpnn_encoder_scalar.cpp:289-321)
//     D1 = h_E W11b^T                     M = 128 slots, N = 128 features
//     G  = GELU(D1 + [W11a h_i + b11] + W11c h_j)
//     G  = GELU(G W12^T + b12)
//     h_E = LN3(h_E + G W13^T + b13)      on slots with a valid neighbour
//   Slots are the A operand here (TMEM lanes), so each slot's 128 features are
//   one TMEM row; the LayerNorm statistics combine the four 32-column parts.
//
//   enc_featurize_tc: edge features -> W_edge -> LN -> W_e, described below.
//
// All are persistent (one CTA per SM, 16 warps).  Weight images arrive by bulk
// copies: the node pass and the featurisation keep theirs resident, the edge
// pass streams its six images through a 3-slot ring and uses the space to
// stage its row gathers.  The next tile's h_E rows are fetched by TMA (a 2-D
// tensor map over this GPU's own h_E, 128-byte swizzle, no multicast) as soon
// as the current tile's first MMA has read them, node terms are gathered while
// MMAs run, and a tile's MMAs are issued by one thread and completion-tracked
// on one mbarrier.  Every wait is bounded.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace hkb {
namespace {

using namespace tc;

constexpr int kEncThreads = 512;
constexpr uint32_t kW128Bytes = 128 * 128 * 2;   // one 128x128 fp16 weight image


// The GELUs here use the fitted tanh form (gelu_tc_x2, max error 2.5e-5)
// on the packed fp32 pipe: every result is rounded to fp16 (4.9e-4 relative)
// or summed with other fitted values, so the exact erf form would buy nothing
// at several times the instructions.

// RBF value f of 16 for the fp16 feature operand: exp(-((d - c_f) / 1.25)^2)
// with c_f = 2 + f * 20/15 and 2 sigma^2 = 1.5625 (the reference's centres and
// width, rbf_scalar.cpp:10-35), by the hardware exponential; the relative
// error (~1e-6) is far below the fp16 rounding of the operand.
__device__ __forceinline__ float rbf_fast(float dist, int f) {
  const float c = 2.0f + (float)f * (20.0f / 15.0f);
  const float dl = dist - c;
  return __expf(-(dl * dl) * (1.0f / 1.5625f));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// fp16 pair of (a, b) or, with lo, of their remainders a - fp16(a), b - fp16(b)
// (exact in fp32): an operand x = hi + lo applied by two MMAs into one
// accumulator carries about twice the fp16 precision.
__device__ __forceinline__ uint32_t pack_h2s(float a, float b, bool lo) {
  if (!lo) return pack_h2(a, b);
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  return pack_h2(a - hf.x, b - hf.y);
}

__device__ __forceinline__ uint32_t idesc_f16(int M, int N) {
  return idesc_bf16(M, N) & ~((7u << 7) | (7u << 10));
}

// h_E tile of `rows` rows from global row `row0` into the SW128 K-major tile
// at `dst` (1024-byte aligned): two TMA boxes, one per 64-column atom; rows
// past the end read as zero.  One thread issues it; `bar` completes when both
// boxes have landed.
__device__ __forceinline__ void tma_rows(unsigned char* dst, const CUtensorMap* map, int64_t row0,
                                         int rows, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, (uint32_t)rows * 256u);
  tma_load_2d(dst, map, 0, (int)row0, bar);
  tma_load_2d(dst + rows * 128, map, 64, (int)row0, bar);
}

__device__ __forceinline__ void load_weights(unsigned char* dst, const unsigned char* const* imgs,
                                             int n, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, (uint32_t)n * kW128Bytes);
  for (int i = 0; i < n; ++i)
    for (uint32_t o = 0; o < kW128Bytes; o += 16384u)
      bulk_g2s(dst + (size_t)i * kW128Bytes + o, imgs[i] + o, 16384u, bar);
}

// ---------------------------------------------------------------------------
// Node-message kernel: 4 residues (192 slots) per tile.
// ---------------------------------------------------------------------------
constexpr int kNodeRes = 4;
constexpr int kNodeSlots = kNodeRes * kK;                  // 192
static_assert(kNodeSlots == kNodeTileRows, "node tile rows");
constexpr uint32_t kNodeTileBytes = kNodeSlots * 256;      // 48 KiB
constexpr uint32_t kNodeOffW = 0;                          // W1b, W2, W1b rem., W2 rem.
constexpr uint32_t kNodeOffB = 4 * kW128Bytes;             // h_E tile
constexpr uint32_t kNodeOffG = kNodeOffB + kNodeTileBytes;
constexpr uint32_t kNodeOffJ = kNodeOffG + kNodeTileBytes; // int [192] rj, float [192] att
constexpr uint32_t kNodeSmem = kNodeOffJ + 2 * kNodeSlots * 4 + 1024;
static_assert(kNodeSmem <= 227 * 1024, "node kernel shared memory");

__global__ void __launch_bounds__(kEncThreads, 1)
    enc_node_tc_kernel(const __grid_constant__ EncNodeTcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  int* SJ = reinterpret_cast<int*>(sm + kNodeOffJ);
  float* SA = reinterpret_cast<float*>(sm + kNodeOffJ + kNodeSlots * 4);
  __shared__ uint64_t bar_w, bar_mma, bar_a;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, rho = warp >> 2;      // feature quadrant, residue of the tile
  const int f = quad * 32 + lane;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int R = p.bv.total_residues;
  const int tiles = (R + kNodeRes - 1) / kNodeRes;

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_a, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    const unsigned char* imgs[4] = {p.W1b, p.W2, p.W1b_lo, p.W2_lo};
    load_weights(sm + kNodeOffW, imgs, 4, &bar_w);
  }
  bool ok = true;
  if (!mbar_wait(&bar_w, 0, p.err)) ok = false;
  uint32_t ph = 0;
  const float b2 = p.b2[f];

  // h_E tiles arrive by TMA; thread kIssuer issues them and the tile's MMAs.
  // It sits outside the threads that fill SJ / SA, so its stall while the
  // tensor pipe accepts the MMAs overlaps their index loads.
  constexpr int kIssuer = kEncThreads - 64;
  static_assert(kIssuer >= kNodeSlots, "MMA issuer outside the SJ / SA threads");
  int t = blockIdx.x;
  uint32_t ph_a = 0;
  bool a_pending = false;   // kIssuer: a tile load not yet waited for
  if (tid == kIssuer && t < tiles) {
    tma_rows(sm + kNodeOffB, &p.map_he, (int64_t)t * kNodeSlots, kNodeSlots, &bar_a);
    a_pending = true;
  }
  for (int it = 0; t < tiles; t += gridDim.x, ++it) {
    if (__syncthreads_or(!ok)) break;
    unsigned char* btile = sm + kNodeOffB;
    if (tid == kIssuer) {
      if (!mbar_wait(&bar_a, ph_a, p.err)) ok = false;
      ph_a ^= 1;
      a_pending = false;
      // D1 = W1b h_E as (hi + remainder) h_E: two MMAs into one accumulator
      tc_fence_after();
      mma_k128(tm, smem_u32(sm + kNodeOffW), smem_u32(btile), kNodeSlots,
               idesc_f16(128, kNodeSlots), false);
      mma_k128(tm, smem_u32(sm + kNodeOffW + 2 * kW128Bytes), smem_u32(btile), kNodeSlots,
               idesc_f16(128, kNodeSlots), true);
      mma_commit(&bar_mma);
    }
    // neighbour rows and attention weights of this tile's slots
    if (tid < kNodeSlots) {
      const int r = t * kNodeRes + tid / kK, k = tid % kK;
      int rj = -1;
      float att = 0.0f;
      if (r < R) {
        const int b = p.bv.res_prot[r];
        const int L = p.bv.prot_len[b];
        const int K = L < kK ? L : kK;
        const int j = k < K ? p.e_idx[(int64_t)r * kK + k] : -1;
        if (j >= 0 && j < L) {
          rj = p.bv.prot_res_off[b] + j;
          att = p.mask[r] * p.mask[rj];
        }
      }
      SJ[tid] = rj;
      SA[tid] = att;
    }
    __syncthreads();
    // node terms of this residue's slots: N_i and the first 16 slots' N_j,
    // gathered while the D1 MMAs run (each 16-slot step loads the next 16)
    const int r = t * kNodeRes + rho;
    const float na = r < R ? p.NAC[(int64_t)r * 256 + f] : 0.0f;
    float ncn[16];
    auto load_nc = [&](int k0, float (&dst)[16]) {
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const int rj = SJ[rho * kK + k0 + k];
        dst[k] = rj >= 0 ? p.NAC[(int64_t)rj * 256 + 128 + f] : 0.0f;
      }
    };
    load_nc(0, ncn);
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    // The h_E tile is free once D1's MMAs have completed: the next tile's rows
    // load during this tile's epilogues.
    const int tn = t + gridDim.x;
    if (tid == kIssuer && tn < tiles) {
      tma_rows(sm + kNodeOffB, &p.map_he, (int64_t)tn * kNodeSlots, kNodeSlots, &bar_a);
      a_pending = true;
    }
    // epilogue 1: G[slot][f] = GELU(D1 + N_i + N_j)  (16-bit stores, B layout),
    // 16 TMEM columns at a time
    unsigned char* G = sm + kNodeOffG;
#pragma unroll
    for (int k0 = 0; k0 < kK; k0 += 16) {
      float ncc[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) ncc[k] = ncn[k];
      if (k0 + 16 < kK) load_nc(k0 + 16, ncn);
      float v[16];
      tmem_ld16(tm + lane_base + (uint32_t)(rho * kK + k0), v);
#pragma unroll
      for (int k = 0; k < 16; k += 2) {
        const int c = rho * kK + k0 + k;
        const int rj0 = SJ[c], rj1 = SJ[c + 1];
        const float nc0 = ncc[k], nc1 = ncc[k + 1];
        const float2 y = gelu_tc_x2(make_float2(v[k] + na + nc0, v[k + 1] + na + nc1));
        *reinterpret_cast<__half*>(G + sw128_offset(c, f, kNodeSlots)) =
            __float2half_rn(rj0 >= 0 ? y.x : 0.0f);
        *reinterpret_cast<__half*>(G + sw128_offset(c + 1, f, kNodeSlots)) =
            __float2half_rn(rj1 >= 0 ? y.y : 0.0f);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == kIssuer) {
      tc_fence_after();
      mma_k128(tm, smem_u32(sm + kNodeOffW + kW128Bytes), smem_u32(G), kNodeSlots,
               idesc_f16(128, kNodeSlots), false);
      mma_k128(tm, smem_u32(sm + kNodeOffW + 3 * kW128Bytes), smem_u32(G), kNodeSlots,
               idesc_f16(128, kNodeSlots), true);
      mma_commit(&bar_mma);
    }
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    // epilogue 2: masked slot sum of GELU(D2 + b2): four interleaved partial
    // sums (slot k goes to k % 4) combined in a fixed order
    {
      // (partials 0,1 and 2,3 as float2 pairs: slots k, k+1 with k % 4 = 0
      // go to pair 0, with k % 4 = 2 to pair 1; a * GELU(x) is one fma of
      // a/2 and twice the GELU, exact scalings by 2)
      float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
      float cnt = 0.0f;
      const float2 b2p = make_float2(b2, b2);
#pragma unroll 1
      for (int k0 = 0; k0 < kK; k0 += 16) {
        float v[16];
        tmem_ld16(tm + lane_base + (uint32_t)(rho * kK + k0), v);
#pragma unroll
        for (int k = 0; k < 16; k += 2) {
          const float a0 = SA[rho * kK + k0 + k], a1 = SA[rho * kK + k0 + k + 1];
          const float2 g2 = gelu2_tc_x2(__fadd2_rn(make_float2(v[k], v[k + 1]), b2p));
          acc[(k >> 1) & 1] = __ffma2_rn(make_float2(0.5f * a0, 0.5f * a1), g2, acc[(k >> 1) & 1]);
          cnt += a0;
          cnt += a1;
        }
      }
      if (r < R) {
        p.S[(int64_t)r * kH + f] = (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
        if (f == 0) p.cnt[r] = cnt;
      }
    }
    tc_fence_before();
  }
  // no TMA load may be in flight when the CTA exits (after an early exit)
  if (tid == kIssuer && a_pending) mbar_wait(&bar_a, ph_a, p.err);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// Edge-update kernel: 128 slots per tile.
// ---------------------------------------------------------------------------
constexpr uint32_t kEdgeTileBytes = 128 * 256;             // 32 KiB
// The six weight images (W11b, W12, W13, each as fp16 value and fp16
// remainder W - hi) stream through a 3-slot ring in the order the MMAs use
// them; a tile consumes ring entries 6i .. 6i+5.  X stages gathered rows so
// that every global load of the pass reads whole rows per warp instruction:
// the neighbour node terms W11c h_j (fp32 [128][128]) while D1 runs, then the
// tile's residual h_E (fp16 value and remainder, [128][128] each) from
// epilogue 1 to epilogue 3, then the LayerNorm output for the store.  A
// thread owns one TMEM row (slot) and 32 columns, so loading its own row
// pieces directly would touch 32 rows per warp instruction.
constexpr int kEdgeRing = 3;
constexpr uint32_t kEdgeOffW = 0;                                   // weight ring
constexpr uint32_t kEdgeOffA = kEdgeRing * kW128Bytes;              // h_E tile (MMA operand)
constexpr uint32_t kEdgeOffG = kEdgeOffA + kEdgeTileBytes;          // GELU operand
constexpr uint32_t kEdgeOffRed = kEdgeOffG;   // float [2][4][128], used when G is free
constexpr uint32_t kEdgeOffX = kEdgeOffG + kEdgeTileBytes;          // 64 KiB staging
constexpr uint32_t kEdgeSmem = kEdgeOffX + 2 * kEdgeTileBytes + 1024;
static_assert(kEdgeSmem <= 227 * 1024, "edge kernel shared memory");

__global__ void __launch_bounds__(kEncThreads, 1)
    enc_edge_tc_kernel(const __grid_constant__ EncEdgeTcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float (*red)[4][128] = reinterpret_cast<float (*)[4][128]>(sm + kEdgeOffRed);
  unsigned char* X = sm + kEdgeOffX;
  __shared__ uint64_t bar_mma, bar_a, bar_w[kEdgeRing];
  // global residue row of each tile row's neighbour (-1: none); [it & 1] is
  // the current tile, the other buffer is filled for the next one
  __shared__ int SJ[2][128];
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;       // slot quadrant, 32-column group
  const int row = quad * 32 + lane;
  const int c0 = cg * 32;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int R = p.bv.total_residues;
  const int64_t SL = (int64_t)R * kK;
  const int64_t tiles = (SL + 127) / 128;

  int64_t t = blockIdx.x;
  if (tid == 0) {
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_a, 1);
    for (int i = 0; i < kEdgeRing; ++i) mbar_init(&bar_w[i], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  // neighbour rows of this CTA's first tile
  if (tid < 128) {
    const int64_t s = t * 128 + tid;
    int rj = -1;
    if (s < SL) {
      const int r = (int)(s / kK), k = (int)(s % kK);
      const int b = p.bv.res_prot[r];
      const int L = p.bv.prot_len[b];
      const int j = k < (L < kK ? L : kK) ? p.e_idx[s] : -1;
      if (j >= 0 && j < L) rj = p.bv.prot_res_off[b] + j;
    }
    SJ[0][tid] = rj;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;

  // weight ring (thread 0): entry j is image j % 6 of this CTA's tile j / 6,
  // in slot j % 3; it is issued once entry j - 3's MMAs have completed.
  const int my_tiles =
      (int)((int64_t)blockIdx.x < tiles ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0);
  const int w_total = my_tiles * 6;
  int w_issued = 0, w_landed = 0;   // entries issued / waited for successfully
  auto w_img = [&](int i) -> const unsigned char* {
    switch (i) {
      case 0: return p.W11b;
      case 1: return p.W11b_lo;
      case 2: return p.W12;
      case 3: return p.W12_lo;
      case 4: return p.W13;
      default: return p.W13_lo;
    }
  };
  auto w_issue = [&](int j) {
    if (j >= w_total) return;
    const int slot = j % kEdgeRing;
    mbar_arrive_expect_tx(&bar_w[slot], kW128Bytes);
    const unsigned char* img = w_img(j % 6);
    for (uint32_t o = 0; o < kW128Bytes; o += 16384u)
      bulk_g2s(sm + kEdgeOffW + slot * kW128Bytes + o, img + o, 16384u, &bar_w[slot]);
    w_issued = j + 1;
  };
  auto w_wait = [&](int j, bool& okf) -> uint32_t {
    const int slot = j % kEdgeRing;
    if (mbar_wait(&bar_w[slot], (uint32_t)((j / kEdgeRing) & 1), p.err)) w_landed = j + 1;
    else okf = false;
    return smem_u32(sm + kEdgeOffW + slot * kW128Bytes);
  };
  if (tid == 0) {
    w_issue(0);
    w_issue(1);
    w_issue(2);
  }
  bool ok = true;
  uint32_t ph = 0;
  const uint32_t idesc = idesc_f16(128, 128);
  unsigned char* G = sm + kEdgeOffG;
  // the next tile's neighbour-index chain (threads 0..127), loaded in three
  // steps spread over the current tile so that no load is waited for
  int nx_e = -1, nx_b = 0, nx_L = 0, nx_off = 0;

  // h_E tiles arrive by TMA (thread 0 issues and waits; only the MMAs read them)
  uint32_t ph_a = 0;
  bool a_pending = false;   // thread 0: a tile load not yet waited for
  if (tid == 0 && t < tiles) {
    tma_rows(sm + kEdgeOffA, &p.map_he, t * 128, 128, &bar_a);
    a_pending = true;
  }
  for (int it = 0; t < tiles; t += gridDim.x, ++it) {
    if (__syncthreads_or(!ok)) break;
    const int j0 = 6 * it;
    const int* sj = SJ[it & 1];
    unsigned char* atile = sm + kEdgeOffA;
    // The tile rows' neighbour terms W11c h_j (512 B per row) into X while the
    // D1 MMAs run: chunk e = tid + 512 i is 16-byte chunk e & 31 of row e >> 5,
    // so each warp instruction reads one whole row; rows without a neighbour
    // are zero-filled.  Issued before the MMAs: thread 0's warp stalls while
    // the tensor pipe accepts them, and these copies are on every warp's path.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + kEncThreads * i;
      const int rr = e >> 5, cc = e & 31;
      const int rj = sj[rr];
      const float* src = p.NAC + (rj >= 0 ? (int64_t)rj * 256 + 128 + cc * 4 : 0);
      cp_async16(X + rr * 512 + ((cc ^ (rr & 7)) << 4), src, rj >= 0);
    }
    cp_async_commit();
    if (tid == 0) {
      if (!mbar_wait(&bar_a, ph_a, p.err)) ok = false;
      ph_a ^= 1;
      a_pending = false;
      // each weight as hi + remainder: two MMAs into one accumulator
      uint32_t w = w_wait(j0, ok);
      tc_fence_after();
      mma_k128(tm, smem_u32(atile), w, 128, idesc, false);
      w = w_wait(j0 + 1, ok);
      tc_fence_after();
      mma_k128(tm, smem_u32(atile), w, 128, idesc, true);
      mma_commit(&bar_mma);
    }
    // this thread's slot; its own node term [W11a h_i + b11] (the slots of a
    // warp span at most two residues, so these loads are near-broadcasts)
    const int64_t s = t * 128 + row;
    const int rj = sj[row];
    float nsum[32];
    {
      const int r = (int)((s < SL ? s : 0) / kK);
      const float4* na = reinterpret_cast<const float4*>(p.NAC + (int64_t)r * 256 + c0);
      float4 a[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) a[q] = na[q];
      cp_async_wait_all();
      __syncthreads();
      const unsigned char* xr = X + row * 512;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 c =
            *reinterpret_cast<const float4*>(xr + (((cg * 8 + q) ^ (row & 7)) << 4));
        nsum[4 * q] = a[q].x + c.x;
        nsum[4 * q + 1] = a[q].y + c.y;
        nsum[4 * q + 2] = a[q].z + c.z;
        nsum[4 * q + 3] = a[q].w + c.w;
      }
    }
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    // D1's MMAs are complete: the h_E tile and entries j0, j0 + 1 are free,
    // so the next tile's rows and weight entries load meanwhile.
    if (tid == 0) {
      w_issue(j0 + 3);
      w_issue(j0 + 4);
    }
    const int64_t tn = t + gridDim.x;
    if (tid == 0 && tn < tiles) {
      tma_rows(atile, &p.map_he, tn * 128, 128, &bar_a);
      a_pending = true;
      // The next tile's remainder rows into L2 a whole tile ahead of its
      // residual staging.
      const int64_t rows = SL - tn * 128 < 128 ? SL - tn * 128 : 128;
      bulk_prefetch_l2(p.h_e_lo + tn * 128 * kH, (uint32_t)(rows * kH * 2));
    }
    if (tid < 128) {   // next tile's index chain, step 1
      nx_e = -1;
      const int64_t sn = tn * 128 + tid;
      if (tn < tiles && sn < SL) {
        nx_b = p.bv.res_prot[(int)(sn / kK)];
        nx_e = p.e_idx[sn];
      }
    }
    // epilogue 1: G = GELU(D1 + N_i + N_j) on this thread's 32 columns
    {
      float v[32];
      tmem_ld32(tm + lane_base + (uint32_t)c0, v);
      uint32_t pk[16];
      if (rj >= 0) {
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float2 y = gelu_tc_x2(__fadd2_rn(make_float2(v[2 * q], v[2 * q + 1]),
                                                 make_float2(nsum[2 * q], nsum[2 * q + 1])));
          pk[q] = pack_h2(y.x, y.y);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) pk[q] = 0u;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(G + sw128_offset(row, c0 + 8 * u, 128)) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      uint32_t w = w_wait(j0 + 2, ok);
      tc_fence_after();
      mma_k128(tm + 128, smem_u32(G), w, 128, idesc, false);
      w = w_wait(j0 + 3, ok);
      tc_fence_after();
      mma_k128(tm + 128, smem_u32(G), w, 128, idesc, true);
      mma_commit(&bar_mma);
    }
    // The tile's residual rows, value then remainder (fp16, 256 B each), into
    // X: every thread has read its node terms (barrier above).  Chunk
    // e = tid + 512 i: array e >> 11, row (e >> 4) & 127, 16-byte chunk e & 15.
    // They land during D2 and epilogue 2 and are waited for before D3.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = tid + kEncThreads * i;
      const int half = e >> 11, rr = (e >> 4) & 127, cc = e & 15;
      const int64_t so = t * 128 + rr;
      const uint16_t* src = (half ? p.h_e_lo : p.h_e) + (so < SL ? so : 0) * kH + cc * 8;
      cp_async16(X + half * kEdgeTileBytes + rr * 256 + ((cc ^ (rr & 15)) << 4), src, so < SL);
    }
    cp_async_commit();
    if (tid < 128 && nx_e >= 0) {   // next tile's index chain, step 2
      nx_L = p.bv.prot_len[nx_b];
      nx_off = p.bv.prot_res_off[nx_b];
    }
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    if (tid == 0) {
      w_issue(j0 + 5);
      w_issue(j0 + 6);
    }
    // epilogue 2: G = GELU(D2 + b12)   (G was consumed by the MMA above)
    {
      float v[32];
      tmem_ld32(tm + lane_base + 128u + (uint32_t)c0, v);
      const float4* b12 = reinterpret_cast<const float4*>(p.b12 + c0);   // warp-uniform
      uint32_t pk[16];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = b12[q];
        const float2 y0 = gelu_tc_x2(make_float2(v[4 * q] + b.x, v[4 * q + 1] + b.y));
        const float2 y1 = gelu_tc_x2(make_float2(v[4 * q + 2] + b.z, v[4 * q + 3] + b.w));
        pk[2 * q] = pack_h2(y0.x, y0.y);
        pk[2 * q + 1] = pack_h2(y1.x, y1.y);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(G + sw128_offset(row, c0 + 8 * u, 128)) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
    }
    cp_async_wait_all();   // residual rows
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      uint32_t w = w_wait(j0 + 4, ok);
      tc_fence_after();
      mma_k128(tm, smem_u32(G), w, 128, idesc, false);
      w = w_wait(j0 + 5, ok);
      tc_fence_after();
      mma_k128(tm, smem_u32(G), w, 128, idesc, true);
      mma_commit(&bar_mma);
    }
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    if (tid == 0) {
      w_issue(j0 + 7);
      w_issue(j0 + 8);
    }
    // epilogue 3: x = h_E + D3 + b13, LayerNorm over the row's 128 features
    // (four 32-column parts held by warps quad, quad+4, quad+8, quad+12)
    {
      float x[32];
      tmem_ld32(tm + lane_base + (uint32_t)c0, x);
      const float2* b13 = reinterpret_cast<const float2*>(p.b13 + c0);   // warp-uniform
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int co = ((cg * 4 + u) ^ (row & 15)) << 4;
        const uint4 hv = *reinterpret_cast<const uint4*>(X + row * 256 + co);
        const uint4 lv = *reinterpret_cast<const uint4*>(X + kEdgeTileBytes + row * 256 + co);
        const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w}, lw[4] = {lv.x, lv.y, lv.z, lv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 h2 = __half22float2(*reinterpret_cast<const __half2*>(&hw[i]));
          const float2 l2 = __half22float2(*reinterpret_cast<const __half2*>(&lw[i]));
          const float2 b = b13[4 * u + i];
          const int c = 8 * u + 2 * i;
          x[c] += (h2.x + l2.x) + b.x;
          x[c + 1] += (h2.y + l2.y) + b.y;
        }
      }
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) sum += x[i];
      // a row's four 32-column parts belong to warps quad, quad+4, quad+8,
      // quad+12: a named barrier over those four suffices
      red[0][cg][row] = sum;
      named_bar_sync(1 + quad, 128);
      const float mean =
          (red[0][0][row] + red[0][1][row] + red[0][2][row] + red[0][3][row]) * (1.0f / 128.0f);
      float sq = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        x[i] -= mean;
        sq += x[i] * x[i];
      }
      red[1][cg][row] = sq;
      named_bar_sync(1 + quad, 128);
      const float var =
          (red[1][0][row] + red[1][1][row] + red[1][2][row] + red[1][3][row]) * (1.0f / 128.0f);
      const float inv = 1.0f / sqrtf(var + kLnEps);
      {
        const float4* gw = reinterpret_cast<const float4*>(p.n3w + c0);   // warp-uniform
        const float4* gb = reinterpret_cast<const float4*>(p.n3b + c0);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 g = gw[q], b = gb[q];
          x[4 * q] = x[4 * q] * inv * g.x + b.x;
          x[4 * q + 1] = x[4 * q + 1] * inv * g.y + b.y;
          x[4 * q + 2] = x[4 * q + 2] * inv * g.z + b.z;
          x[4 * q + 3] = x[4 * q + 3] * inv * g.w + b.w;
        }
      }
      uint32_t pv[16], pl[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const __half2 h = __floats2half2_rn(x[2 * q], x[2 * q + 1]);
        const float2 hf = __half22float2(h);
        pv[q] = *reinterpret_cast<const uint32_t*>(&h);
        const __half2 l = __floats2half2_rn(x[2 * q] - hf.x, x[2 * q + 1] - hf.y);
        pl[q] = *reinterpret_cast<const uint32_t*>(&l);
      }
      __syncthreads();   // every read of the residual rows in X is done
      // Value and remainder rows staged in X (same layout as the residual),
      // then copied out as whole rows; rows without a valid neighbour are not
      // written (edge_update keeps them).
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int co = ((cg * 4 + u) ^ (row & 15)) << 4;
        *reinterpret_cast<uint4*>(X + row * 256 + co) =
            make_uint4(pv[4 * u], pv[4 * u + 1], pv[4 * u + 2], pv[4 * u + 3]);
        *reinterpret_cast<uint4*>(X + kEdgeTileBytes + row * 256 + co) =
            make_uint4(pl[4 * u], pl[4 * u + 1], pl[4 * u + 2], pl[4 * u + 3]);
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = tid + kEncThreads * i;
        const int half = e >> 11, rr = (e >> 4) & 127, cc = e & 15;
        const int64_t so = t * 128 + rr;
        uint16_t* out = half ? p.h_e_lo : p.h_e_out;
        if (so < SL && sj[rr] >= 0)
          *reinterpret_cast<uint4*>(out + so * kH + cc * 8) = *reinterpret_cast<const uint4*>(
              X + half * kEdgeTileBytes + rr * 256 + ((cc ^ (rr & 15)) << 4));
      }
    }
    // next tile's index chain, step 3: its neighbour rows, read after the
    // barriers at the top of the next iteration
    if (tid < 128) {
      int rjn = -1;
      if (nx_e >= 0) {
        const int kn = (int)((tn * 128 + tid) % kK);
        if (kn < (nx_L < kK ? nx_L : kK) && nx_e < nx_L) rjn = nx_off + nx_e;
      }
      SJ[(it + 1) & 1][tid] = rjn;
    }
    tc_fence_before();
  }
  cp_async_wait_all();
  // Drain: no bulk or TMA copy may be in flight when the CTA exits (entries
  // issued but not waited for after an early exit).
  if (tid == 0) {
    for (int j = w_landed; j < w_issued; ++j)
      mbar_wait(&bar_w[j % kEdgeRing], (uint32_t)((j / kEdgeRing) & 1), p.err);
    if (a_pending) mbar_wait(&bar_a, ph_a, p.err);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// Featurisation kernel: 128 slots per tile (inverse_fold_scalar.cpp:236-279,
// edge_rbf_features_scalar.cpp:45-137):
//   f   = [W_pos[:, class(i - j)] + b_pos (16) | RBF of 25 atom pairs (400) | 0 (32)]
//   E   = f W_edge^T          K = 448 as four chunks of 2, 2, 2 and 1 64-column atoms
//   h_E = LN_e(E) W_e^T + b_e   (fp16 out)
// Features are computed straight into the SW128 operand, each once, as fp16
// value and fp16 remainder, so the [R*48, 416] feature matrix never exists
// in HBM.
// ---------------------------------------------------------------------------
constexpr uint32_t kAtomBytes = 128 * 128;                    // 128 rows x 64 fp16
constexpr uint32_t kFeatOffWedge = 0;                         // 7 atoms
constexpr uint32_t kFeatOffWe = 7 * kAtomBytes;               // 2 atoms
constexpr uint32_t kFeatOffA = kFeatOffWe + kW128Bytes;       // 4 atoms: features / LN operand
constexpr uint32_t kFeatOffRow = kFeatOffA + 4 * kAtomBytes;  // int [3][128]
constexpr uint32_t kFeatOffRed = kFeatOffRow + 3 * 128 * 4;   // float [2][4][128]
constexpr uint32_t kFeatSmem = kFeatOffRed + 2 * 4 * 128 * 4 + 1024;

// One RBF item: the 16 values of atom pair p for tile row `row`, computed
// once and stored as fp16 values at local column `col` of the K chunk
// (operand atoms 0-1) and as fp16 remainders at `col` + 128 (atoms 2-3).
__device__ __forceinline__ void feat_pair_item(unsigned char* A, int row, int p, int col,
                                               const int* SR, const int* SJ,
                                               const EncFeatTcArgs& a) {
  uint32_t ph[8] = {0, 0, 0, 0, 0, 0, 0, 0}, pl[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int r = SR[row], rj = SJ[row];
  if (rj >= 0) {
    const int ai = c_pairs[p][0], aj = c_pairs[p][1];
    if (a.src[(int64_t)r * 5 + ai] && a.src[(int64_t)rj * 5 + aj]) {
      const float dist =
          pair_distance(a.coords + ((int64_t)r * 5 + ai) * 3, a.coords + ((int64_t)rj * 5 + aj) * 3);
#pragma unroll
      for (int f = 0; f < 8; ++f) {
        const float x0 = rbf_fast(dist, 2 * f), x1 = rbf_fast(dist, 2 * f + 1);
        ph[f] = pack_h2s(x0, x1, false);
        pl[f] = pack_h2s(x0, x1, true);
      }
    }
  }
  *reinterpret_cast<uint4*>(A + sw128_offset(row, col, 128)) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
  *reinterpret_cast<uint4*>(A + sw128_offset(row, col + 8, 128)) =
      make_uint4(ph[4], ph[5], ph[6], ph[7]);
  *reinterpret_cast<uint4*>(A + sw128_offset(row, col + 128, 128)) =
      make_uint4(pl[0], pl[1], pl[2], pl[3]);
  *reinterpret_cast<uint4*>(A + sw128_offset(row, col + 136, 128)) =
      make_uint4(pl[4], pl[5], pl[6], pl[7]);
}

__global__ void __launch_bounds__(kEncThreads, 1)
    enc_featurize_tc_kernel(EncFeatTcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  int* SR = reinterpret_cast<int*>(sm + kFeatOffRow);    // residue of the row (-1: none)
  int* SJ = SR + 128;                                    // neighbour residue (-1: invalid)
  int* SC = SR + 256;                                    // positional class (-1: none)
  float (*red)[4][128] = reinterpret_cast<float (*)[4][128]>(sm + kFeatOffRed);
  unsigned char* A = sm + kFeatOffA;
  __shared__ uint64_t bar_w, bar_mma;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;
  const int row = quad * 32 + lane;
  const int c0 = cg * 32;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int R = p.bv.total_residues;
  const int64_t SL = (int64_t)R * kK;
  const int64_t tiles = (SL + 127) / 128;

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_mma, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar_w, 7 * kAtomBytes + kW128Bytes);
    for (uint32_t o = 0; o < 7 * kAtomBytes; o += 16384u)
      bulk_g2s(sm + kFeatOffWedge + o, p.Wedge + o, 16384u, &bar_w);
    for (uint32_t o = 0; o < kW128Bytes; o += 16384u)
      bulk_g2s(sm + kFeatOffWe + o, p.We + o, 16384u, &bar_w);
  }
  bool ok = true;
  if (!mbar_wait(&bar_w, 0, p.err)) ok = false;
  uint32_t ph = 0;
  const uint32_t idesc = idesc_f16(128, 128);

  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    if (__syncthreads_or(!ok)) break;
    if (tid < 128) {
      const int64_t s = t * 128 + tid;
      int r = -1, rj = -1, cls = -1;
      if (s < SL) {
        r = (int)(s / kK);
        const int k = (int)(s % kK);
        const int b = p.bv.res_prot[r];
        const int off = p.bv.prot_res_off[b];
        const int L = p.bv.prot_len[b];
        const int K = L < kK ? L : kK;
        const int j = k < K ? p.e_idx[s] : -1;
        if (j >= 0 && j < L) {
          rj = off + j;
          int o = (r - off) - j;
          o = o < -32 ? -32 : (o > 32 ? 32 : o);
          cls = o + 32;
        }
      }
      SR[tid] = r;
      SJ[tid] = rj;
      SC[tid] = cls;
    }
    __syncthreads();
    // The 448 feature columns (positional block 0-15, pairs 0-24 at 16-415,
    // zeros 416-447) in four K chunks of 128, 128, 128 and 64 columns
    // (pairs 0-6, 7-14, 15-22, 23-24).  Each feature is computed once and
    // stored as its fp16 value (operand atoms 0-1) and fp16 remainder (atoms
    // 2-3); the chunk's value and remainder products accumulate into E.
    for (int c = 0; c < 4; ++c) {
      const int p0 = c == 0 ? 0 : 8 * c - 1;           // first pair of the chunk
      const int np = c == 0 ? 7 : (c == 3 ? 2 : 8);    // pairs in the chunk
      const int npos = c == 0 ? 256 : 0;               // 128 rows x 2 positional halves
      const int nzero = c == 3 ? 4 * 128 : 0;          // 128 rows x 4 zero 8-column parts
      const int items = npos + np * 128 + nzero;
      for (int m = tid; m < items; m += kEncThreads) {
        if (m < npos) {
          const int rw = m >> 1, h = (m & 1) * 8;
          const int cls = SC[rw];
          uint32_t vh[4] = {0, 0, 0, 0}, vl[4] = {0, 0, 0, 0};
          if (cls >= 0) {
#pragma unroll
            for (int d = 0; d < 4; ++d) {
              const int d0 = h + 2 * d;
              const float x0 = p.pos_w[d0 * kPosClasses + cls] + p.pos_b[d0];
              const float x1 = p.pos_w[(d0 + 1) * kPosClasses + cls] + p.pos_b[d0 + 1];
              vh[d] = pack_h2s(x0, x1, false);
              vl[d] = pack_h2s(x0, x1, true);
            }
          }
          *reinterpret_cast<uint4*>(A + sw128_offset(rw, h, 128)) =
              make_uint4(vh[0], vh[1], vh[2], vh[3]);
          *reinterpret_cast<uint4*>(A + sw128_offset(rw, h + 128, 128)) =
              make_uint4(vl[0], vl[1], vl[2], vl[3]);
        } else if (m < npos + np * 128) {
          const int q = m - npos, rw = q & 127, pr = p0 + (q >> 7);
          feat_pair_item(A, rw, pr, 16 + 16 * pr - 128 * c, SR, SJ, p);
        } else {
          const int q = m - npos - np * 128, rw = q >> 2, u = q & 3;
          *reinterpret_cast<uint4*>(A + sw128_offset(rw, 32 + 8 * u, 128)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(A + sw128_offset(rw, 160 + 8 * u, 128)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        const uint32_t wb = smem_u32(sm + kFeatOffWedge) + (uint32_t)(2 * c) * kAtomBytes;
        const int ksteps = c == 3 ? 4 : 8;
        for (int half = 0; half < 2; ++half)
          for (int kk = 0; kk < ksteps; ++kk) {
            const uint32_t o = (uint32_t)(kk >> 2) * kAtomBytes + (uint32_t)(kk & 3) * 32u;
            mma_bf16(tm, sw128_desc(smem_u32(A) + (uint32_t)half * 2u * kAtomBytes + o),
                     sw128_desc(wb + o), idesc, (c > 0 || half > 0 || kk > 0) ? 1u : 0u);
          }
        mma_commit(&bar_mma);
      }
      if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
      ph ^= 1;
      tc_fence_after();
    }
    // LayerNorm of the 128-wide edge row (four 32-column parts) -> fp16 operand
    {
      float x[32];
      tmem_ld32(tm + lane_base + (uint32_t)c0, x);
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) sum += x[i];
      red[0][cg][row] = sum;
      __syncthreads();
      const float mean =
          (red[0][0][row] + red[0][1][row] + red[0][2][row] + red[0][3][row]) * (1.0f / 128.0f);
      float sq = 0.0f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        x[i] -= mean;
        sq += x[i] * x[i];
      }
      red[1][cg][row] = sq;
      __syncthreads();
      const float var =
          (red[1][0][row] + red[1][1][row] + red[1][2][row] + red[1][3][row]) * (1.0f / 128.0f);
      const float inv = 1.0f / sqrtf(var + kLnEps);
#pragma unroll
      for (int i = 0; i < 32; ++i) x[i] = x[i] * inv * p.ln_w[c0 + i] + p.ln_b[c0 + i];
      // LN_e(E) as fp16 (pass 0), then its fp16 remainder (pass 1), each
      // times W_e into one accumulator
      for (int pass = 0; pass < 2; ++pass) {
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) pk[q] = pack_h2s(x[2 * q], x[2 * q + 1], pass == 1);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          *reinterpret_cast<uint4*>(A + sw128_offset(row, c0 + 8 * u, 128)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
          tc_fence_after();
          mma_k128(tm + 128, smem_u32(A), smem_u32(sm + kFeatOffWe), 128, idesc, pass == 1);
          mma_commit(&bar_mma);
        }
        if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
        ph ^= 1;
        tc_fence_after();
      }
    }
    {
      float v[32];
      tmem_ld32(tm + lane_base + 128u + (uint32_t)c0, v);
      const float4* wb = reinterpret_cast<const float4*>(p.We_b + c0);   // warp-uniform
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = wb[q];
        v[4 * q] += b.x;
        v[4 * q + 1] += b.y;
        v[4 * q + 2] += b.z;
        v[4 * q + 3] += b.w;
      }
      // h_E value, then remainder, through the operand buffer (free: the
      // W_e products have completed) so each warp instruction stores two
      // contiguous 256-byte rows
      uint32_t ph[16], pl[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        ph[q] = pack_h2s(v[2 * q], v[2 * q + 1], false);
        pl[q] = pack_h2s(v[2 * q], v[2 * q + 1], true);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint32_t* pk = half ? pl : ph;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int cc = cg * 4 + u;
          *reinterpret_cast<uint4*>(A + row * 256 + ((cc ^ (row & 15)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
        __syncthreads();
        uint16_t* out = half ? p.h_e_lo : p.h_e;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int idx = tid + kEncThreads * i;
          const int rr = idx >> 4, cc = idx & 15;
          const int64_t so = t * 128 + rr;
          if (so < SL)
            *reinterpret_cast<uint4*>(out + so * kH + cc * 8) =
                *reinterpret_cast<const uint4*>(A + rr * 256 + ((cc ^ (rr & 15)) << 4));
        }
        __syncthreads();
      }
    }
    tc_fence_before();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// Decoder slot tables: PE_l = h_E W1b_l^T + PVenc_l[j] (l = 0..2, fp16 out) in
// one pass over h_E -- the three decoder layers' h_E input blocks
// (decoder_layer_scalar.cpp:26-69 split by input block) share the A tile, and
// the epilogue adds the slot neighbour's fp16 W1d_l h_enc row (gathered while
// the MMAs run) before the single rounding to fp16.
// ---------------------------------------------------------------------------
constexpr uint32_t kTabOffW = 0;                            // 3 images
constexpr uint32_t kTabOffA = 3 * kW128Bytes;               // 2 h_E tiles
// X: one layer's gathered PVenc rows [128][256 B], then that layer's output
// rows [128][256 B] (16-bit), so that gathers and stores move whole rows
constexpr uint32_t kTabOffX = kTabOffA + 2 * kEdgeTileBytes;
constexpr uint32_t kTabSmem = kTabOffX + 2 * kEdgeTileBytes + 1024;
static_assert(kTabSmem <= 227 * 1024, "table kernel shared memory");

__global__ void __launch_bounds__(kEncThreads, 1)
    dec_tables_tc_kernel(const __grid_constant__ DecTablesTcArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ uint64_t bar_w, bar_mma, bar_a[2];
  __shared__ int SJ[128];   // global residue row of each tile row's neighbour (-1: none)
  __shared__ uint32_t tmem_base;
  unsigned char* X = sm + kTabOffX;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;
  const int row = quad * 32 + lane;
  const int c0 = cg * 32;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int64_t SL = p.rows;
  const int64_t tiles = (SL + 127) / 128;

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_a[0], 1);
    mbar_init(&bar_a[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    const unsigned char* imgs[3] = {p.W[0], p.W[1], p.W[2]};
    load_weights(sm + kTabOffW, imgs, 3, &bar_w);
  }
  bool ok = true;
  if (!mbar_wait(&bar_w, 0, p.err)) ok = false;
  uint32_t ph = 0;
  const uint32_t idesc = idesc_f16(128, 128);

  // h_E tiles arrive by TMA into two buffers, one tile ahead (thread 0 issues
  // and waits; only the MMAs read them)
  int64_t t = blockIdx.x;
  uint32_t ph_a = 0;     // bit b: phase parity of bar_a[b]
  int a_pending = 0;     // bit b: a load into buffer b not yet waited for
  if (tid == 0 && t < tiles) {
    tma_rows(sm + kTabOffA, &p.map_he, t * 128, 128, &bar_a[0]);
    a_pending = 1;
  }
  for (int it = 0; t < tiles; t += gridDim.x, ++it) {
    if (__syncthreads_or(!ok)) break;
    const int buf = it & 1;
    unsigned char* atile = sm + kTabOffA + buf * kEdgeTileBytes;
    const int64_t tn = t + gridDim.x;
    if (tid == 0) {
      // next tile into the other buffer (its MMAs completed last iteration)
      if (tn < tiles) {
        tma_rows(sm + kTabOffA + (buf ^ 1) * kEdgeTileBytes, &p.map_he, tn * 128, 128,
                 &bar_a[buf ^ 1]);
        a_pending |= 1 << (buf ^ 1);
      }
      if (!mbar_wait(&bar_a[buf], (ph_a >> buf) & 1u, p.err)) ok = false;
      ph_a ^= 1u << buf;
      a_pending &= ~(1 << buf);
      tc_fence_after();
      for (int l = 0; l < 3; ++l)
        mma_k128(tm + 128u * l, smem_u32(atile), smem_u32(sm + kTabOffW + l * kW128Bytes), 128,
                 idesc, false);
      mma_commit(&bar_mma);
    }
    // neighbour residue row of each tile row (-1: no neighbour)
    if (tid < 128) {
      const int64_t s = t * 128 + tid;
      int rj = -1;
      if (s < SL) {
        const int r = (int)(s / kK), k = (int)(s % kK);
        const int b = p.bv.res_prot[r];
        const int L = p.bv.prot_len[b];
        const int j = k < (L < kK ? L : kK) ? p.e_idx[s] : -1;
        if (j >= 0 && j < L) rj = p.bv.prot_res_off[b] + j;
      }
      SJ[tid] = rj;
    }
    __syncthreads();
    // layer l's PVenc rows of the tile's neighbours into X[0, 32 KiB): chunk
    // e = tid + 512 i is 16-byte chunk e & 15 of row e >> 4, so a warp
    // instruction reads two whole rows; rows without a neighbour are zero
    auto stage_pv = [&](int l) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e = tid + kEncThreads * i;
        const int rr = e >> 4, cc = e & 15;
        const int rj = SJ[rr];
        const uint16_t* src = p.PVenc[l] + (rj >= 0 ? (int64_t)rj * kH + cc * 8 : 0);
        cp_async16(X + rr * 256 + ((cc ^ (rr & 15)) << 4), src, rj >= 0);
      }
      cp_async_commit();
    };
    stage_pv(0);
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
    for (int l = 0; l < 3; ++l) {
      cp_async_wait_all();
      __syncthreads();   // layer l's rows landed; layer l-1's copy-out is done
      {
        float v[32];
        tmem_ld32(tm + lane_base + 128u * l + (uint32_t)c0, v);
        uint32_t pk[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int co = ((cg * 4 + u) ^ (row & 15)) << 4;
          const uint4 ev = *reinterpret_cast<const uint4*>(X + row * 256 + co);
          const uint32_t ew[4] = {ev.x, ev.y, ev.z, ev.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 e = __half22float2(*reinterpret_cast<const __half2*>(&ew[i]));
            const int q = 4 * u + i;
            pk[q] = pack_h2(v[2 * q] + e.x, v[2 * q + 1] + e.y);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int co = ((cg * 4 + u) ^ (row & 15)) << 4;
          *reinterpret_cast<uint4*>(X + kEdgeTileBytes + row * 256 + co) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      __syncthreads();   // every PVenc read of layer l and every output write are done
      if (l < 2) stage_pv(l + 1);
      // layer l's table rows, copied out as whole rows
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e = tid + kEncThreads * i;
        const int rr = e >> 4, cc = e & 15;
        const int64_t so = t * 128 + rr;
        if (so < SL)
          *reinterpret_cast<uint4*>(p.out[l] + so * kH + cc * 8) = *reinterpret_cast<const uint4*>(
              X + kEdgeTileBytes + rr * 256 + ((cc ^ (rr & 15)) << 4));
      }
    }
    tc_fence_before();
  }
  // no TMA load may be in flight when the CTA exits (after an early exit)
  if (tid == 0)
    for (int b = 0; b < 2; ++b)
      if ((a_pending >> b) & 1) mbar_wait(&bar_a[b], (ph_a >> b) & 1u, p.err);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 512);
}

}  // namespace

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's cuTensorMapEncodeTiled, looked up once through the runtime (no
// link against libcuda).
EncodeTiledFn encode_tiled() {
  static const EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}
}  // namespace

bool make_rows_tensor_map(CUtensorMap* map, const uint16_t* base, int64_t rows, int box_rows) {
  const EncodeTiledFn fn = encode_tiled();
  if (!fn || !base || rows <= 0 || rows > 0x7FFFFFFF || box_rows <= 0 || box_rows > 256) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)kH, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kH * 2};   // bytes between rows
  const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};  // 64 fp16 = one 128-byte swizzle span
  const cuuint32_t estride[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(base), dims, strides,
            box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void launch_enc_node_tc(cudaStream_t st, const EncNodeTcArgs& p, int num_sms) {
  const int tiles = (p.bv.total_residues + kNodeRes - 1) / kNodeRes;
  if (tiles <= 0) return;
  ensure_dynamic_smem((const void*)enc_node_tc_kernel, (int)kNodeSmem);
  const int grid = tiles < num_sms ? tiles : num_sms;
  enc_node_tc_kernel<<<grid, kEncThreads, kNodeSmem, st>>>(p);
}

void launch_enc_featurize_tc(cudaStream_t st, const EncFeatTcArgs& p, int num_sms) {
  const int64_t tiles = ((int64_t)p.bv.total_residues * kK + 127) / 128;
  if (tiles <= 0) return;
  ensure_dynamic_smem((const void*)enc_featurize_tc_kernel, (int)kFeatSmem);
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  enc_featurize_tc_kernel<<<grid, kEncThreads, kFeatSmem, st>>>(p);
}

void launch_dec_tables_tc(cudaStream_t st, const DecTablesTcArgs& p, int num_sms) {
  const int64_t tiles = (p.rows + 127) / 128;
  if (tiles <= 0) return;
  ensure_dynamic_smem((const void*)dec_tables_tc_kernel, (int)kTabSmem);
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  dec_tables_tc_kernel<<<grid, kEncThreads, kTabSmem, st>>>(p);
}

void launch_enc_edge_tc(cudaStream_t st, const EncEdgeTcArgs& p, int num_sms) {
  const int64_t tiles = ((int64_t)p.bv.total_residues * kK + 127) / 128;
  if (tiles <= 0) return;
  ensure_dynamic_smem((const void*)enc_edge_tc_kernel, (int)kEdgeSmem);
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  enc_edge_tc_kernel<<<grid, kEncThreads, kEdgeSmem, st>>>(p);
}

}  // namespace hkb
