// fp32 (parity-mode) kernels of the ProteinMPNN v_48_020 design engine:
// featurisation (bit-exact CA kNN, atom-pair RBF + positional edge features),
// the encoder and teacher-forced decoder as row/slot kernels around a tiled
// SIMT GEMM, and the fused persistent autoregressive decode kernel.
//
// Layout in HBM (R residues over all proteins of a call, Q = sum S_b L_b rows):
//   e_idx   i32 [R,48]      protein-local neighbour index, -1 past K_b
//   h_E     f32 [R,48,128]  (slots k >= K_b are zero)
//   h_V     f32 [R,128]
//   rows of the decoder are (sequence, residue) pairs; a sequence's L_b rows
//   are contiguous.
#include "common.cuh"
#include "kernels.hpp"

#include <algorithm>
#include <mutex>

namespace hkb {

void ensure_dynamic_smem(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  // A fixed table (no heap allocation: the allocation-free entry point runs
  // through here too).  Past its capacity the attribute is simply set again.
  struct Entry {
    int dev;
    const void* func;
    int bytes;
  };
  constexpr int kCap = 512;
  static Entry done[kCap];
  static int n_done = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_done; ++i)
    if (done[i].dev == dev && done[i].func == func && done[i].bytes == bytes) return;
  cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (n_done < kCap) done[n_done++] = {dev, func, bytes};
}

namespace {

__device__ __forceinline__ void set_err(unsigned int* err, unsigned int bit) {
  if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------------------
// Tiled SIMT GEMM: 64x64 output tile per 256-thread block, 4x4 per thread,
// K staged 16 at a time through shared memory.
// ---------------------------------------------------------------------------
template <int ACT>
__global__ void __launch_bounds__(256) gemm_f32_kernel(
    int64_t M, int N, int K, const float* __restrict__ A, int lda,
    const float* __restrict__ B, int ldb, const float* __restrict__ bias,
    float* __restrict__ C, int ldc) {
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * 64;
  const int n0 = blockIdx.y * 64;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 1024; e += 256) {
      const int r = e >> 4, c = e & 15;
      const int64_t gm = m0 + r;
      const int gk = k0 + c;
      As[c][r] = (gm < M && gk < K) ? A[gm * lda + gk] : 0.0f;
    }
    for (int e = threadIdx.x; e < 1024; e += 256) {
      const int r = e >> 6, c = e & 63;
      const int gk = k0 + r, gn = n0 + c;
      Bs[r][c] = (gk < K && gn < N) ? B[(int64_t)gk * ldb + gn] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float v = acc[i][j] + (bias ? bias[gn] : 0.0f);
      if (ACT == 1) v = gelu_as(v);
      C[gm * ldc + gn] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// fp32 GEMM on the packed fp32 pipe for N a multiple of 128 and K of 32:
// C[M,N] = act(A[M,K] . B[K,N] + bias[N]).  128x128 output tile per
// 256-thread block (two blocks per SM); thread (tx, ty) = (tid % 16,
// tid / 16) owns rows 8 ty .. 8 ty + 7 and columns 8 tx .. 8 tx + 7, as
// float2 column pairs updated by fma.rn.f32x2.  K advances 32 at a time
// through two shared-memory stages filled by cp.async (the next slab loads
// while the current one is multiplied); A stays row-major in shared memory
// and a thread reads two consecutive k of each of its rows at once.  Each
// output is one fp32 fma chain in k order (one rounding per term, as the
// scalar kernel), then bias, then the activation.
// ---------------------------------------------------------------------------
constexpr int kG2Tile = 128;
constexpr int kG2K = 32;
constexpr int kG2APitch = kG2K + 4;   // floats per As row: 144 B, 16-byte aligned
constexpr size_t kG2Smem = (size_t)2 * (kG2Tile * kG2APitch + kG2K * kG2Tile) * sizeof(float);

template <int ACT, bool OUT16>
__global__ void __launch_bounds__(256, 2) gemm_f32x2_kernel(
    int64_t M, int K, const float* __restrict__ A, int lda, const float* __restrict__ B, int ldb,
    const float* __restrict__ bias, void* __restrict__ C, int ldc) {
  extern __shared__ __align__(16) float g2_smem[];
  float (*As)[kG2Tile][kG2APitch] = reinterpret_cast<float (*)[kG2Tile][kG2APitch]>(g2_smem);
  float (*Bs)[kG2K][kG2Tile] =
      reinterpret_cast<float (*)[kG2K][kG2Tile]>(g2_smem + 2 * kG2Tile * kG2APitch);
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * kG2Tile;
  const int n0 = blockIdx.y * kG2Tile;
  // One slab: A 128 rows x 32 k and B 32 rows x 128 n, 1024 16-byte chunks
  // each.  Thread chunk q (0..3) of A is row tid / 8 + 32 q, k 4 (tid % 8);
  // of B row tid / 32 + 8 q, n 4 (tid % 32).  Rows of A past M are
  // zero-filled.
  const int ar = tid >> 3, ak = (tid & 7) * 4;
  const int bk = tid >> 5, bn = (tid & 31) * 4;
  const float* a_base = A + (m0 + ar) * lda + ak;
  const float* b_base = B + (int64_t)bk * ldb + n0 + bn;
  auto load = [&](int k0, int stage) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const bool ok = m0 + ar + 32 * q < M;
      cp_async16(&As[stage][ar + 32 * q][ak], ok ? a_base + (int64_t)(32 * q) * lda + k0 : A, ok);
      cp_async16(&Bs[stage][bk + 8 * q][bn], b_base + (int64_t)(k0 + 8 * q) * ldb, true);
    }
    cp_async_commit();
  };
  float2 acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.0f, 0.0f);

  const int slabs = K / kG2K;
  load(0, 0);
  for (int t = 0; t < slabs; ++t) {
    const int cur = t & 1;
    if (t + 1 < slabs) {
      load((t + 1) * kG2K, cur ^ 1);
      cp_async_wait_one();
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
#pragma unroll 1   // (full unrolling hoists the next step's loads and spills)
    for (int k2 = 0; k2 < kG2K; k2 += 2) {
      float2 a2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) a2[i] = *reinterpret_cast<const float2*>(&As[cur][ty * 8 + i][k2]);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k2 + u][tx * 8]);
        const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k2 + u][tx * 8 + 4]);
        const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                              make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a = u == 0 ? a2[i].x : a2[i].y;
          const float2 ai = make_float2(a, a);
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = __ffma2_rn(ai, bv[j], acc[i][j]);
        }
      }
    }
    __syncthreads();   // stage cur is refilled by the next iteration's load
  }
  float bb[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) bb[j] = bias ? bias[n0 + tx * 8 + j] : 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + ty * 8 + i;
    if (gm >= M) continue;
    float v[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = acc[i][j].x + bb[2 * j];
      v[2 * j + 1] = acc[i][j].y + bb[2 * j + 1];
    }
    if (ACT == 1) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = gelu_as(v[j]);
    }
    if constexpr (OUT16) {
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 p = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
        h[j] = *reinterpret_cast<const uint32_t*>(&p);
      }
      *reinterpret_cast<uint4*>(static_cast<__half*>(C) + gm * ldc + n0 + tx * 8) =
          make_uint4(h[0], h[1], h[2], h[3]);
    } else {
      float* c = static_cast<float*>(C) + gm * ldc + n0 + tx * 8;
      *reinterpret_cast<float4*>(c) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(c + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// ---------------------------------------------------------------------------
// CA kNN, one block per query residue.  Reference semantics
// (cpp/primitives/compute/knn_scalar.cpp:72-168 as configured by
// cpp/modules/mpnn/inverse_fold_scalar.cpp:211-234): d^2 = dx^2 + dy^2 + dz^2
// + 1e-6 in that order with separate roundings; pairs with an invalid residue
// take the row maximum over valid targets; the K smallest by (d^2, index)
// survive -- strict-less insertion keeps the earlier index on ties.  Each
// candidate's rank is counted directly against the packed (d^2 bits, index)
// keys, which is exact because d^2 >= 0 orders like its IEEE bit pattern.
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool residue_valid(const uint8_t* src, int r) {
  const uint8_t* s = src + (int64_t)r * 5;
  return s[0] && s[1] && s[2] && s[3];
}

__device__ __forceinline__ float sqdist_floor(float qx, float qy, float qz,
                                              float tx, float ty, float tz) {
  const float dx = __fsub_rn(qx, tx), dy = __fsub_rn(qy, ty), dz = __fsub_rn(qz, tz);
  float s = __fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy));
  s = __fadd_rn(s, __fmul_rn(dz, dz));
  return __fadd_rn(s, 1.0e-6f);
}

__device__ __forceinline__ void load_ca(const float* coords, const uint8_t* src,
                                        int r, float& x, float& y, float& z) {
  if (src[(int64_t)r * 5 + 1]) {
    const float* c = coords + ((int64_t)r * 5 + 1) * 3;
    x = c[0];
    y = c[1];
    z = c[2];
  } else {
    x = y = z = 0.0f;
  }
}

__global__ void __launch_bounds__(256) knn_kernel(
    BatchView bv, const float* __restrict__ coords,
    const uint8_t* __restrict__ src, int* __restrict__ e_idx,
    float* __restrict__ d2out, float* __restrict__ mask, unsigned int* err) {
  extern __shared__ unsigned long long keys[];
  __shared__ float red[8];
  const int r = blockIdx.x;
  const int b = bv.res_prot[r];
  const int off = bv.prot_res_off[b];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  const bool vq = residue_valid(src, r);
  float qx, qy, qz;
  load_ca(coords, src, r, qx, qy, qz);
  float rmax = 1.0e-6f;
  if (vq) {
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
      if (!residue_valid(src, off + j)) continue;
      float tx, ty, tz;
      load_ca(coords, src, off + j, tx, ty, tz);
      rmax = fmaxf(rmax, sqdist_floor(qx, qy, qz, tx, ty, tz));
    }
  }
  rmax = warp_max(rmax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = rmax;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    red[0] = m;
  }
  __syncthreads();
  rmax = red[0];
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    float d = rmax;
    if (vq && residue_valid(src, off + j)) {
      float tx, ty, tz;
      load_ca(coords, src, off + j, tx, ty, tz);
      d = sqdist_floor(qx, qy, qz, tx, ty, tz);
    }
    keys[j] = ((unsigned long long)__float_as_uint(d) << 32) | (unsigned int)j;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < L; j += blockDim.x) {
    const unsigned long long mine = keys[j];
    int rank = 0;
    for (int m = 0; m < L; ++m) rank += keys[m] < mine ? 1 : 0;
    if (rank < K) {
      e_idx[(int64_t)r * kK + rank] = j;
      if (d2out) d2out[(int64_t)r * kK + rank] = __uint_as_float((unsigned int)(mine >> 32));
    }
  }
  for (int k = K + threadIdx.x; k < kK; k += blockDim.x) {
    e_idx[(int64_t)r * kK + k] = -1;
    if (d2out) d2out[(int64_t)r * kK + k] = 0.0f;
  }
  if (threadIdx.x == 0) mask[r] = vq ? 1.0f : 0.0f;
  (void)err;
}

// ---------------------------------------------------------------------------
// Edge features [R*48, 416]: 16 positional values W_pos[:, class] + b_pos with
// class = clamp(i - j, -32, 32) + 32 (single chain, array positions:
// cpp/modules/mpnn/edge_rbf_features_scalar.cpp:45-76), then per atom pair
// 16 Gaussian RBFs of sqrt(|x_j - x_i|^2 + 1e-6) on centres linspace(2, 22),
// sigma = 20 / (16 / sqrt(1/2)), zero when either atom is missing
// (cpp/primitives/compute/atom_pair_distance_scalar.cpp:122-164,
//  cpp/primitives/compute/rbf_scalar.cpp:10-35).
// The 25 (query atom, neighbour atom) slot pairs follow the reference's table
// (atom_pair_distance_scalar.cpp:21-72); slot order N=0 CA=1 C=2 O=3 CB=4.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256) edge_features_kernel(
    BatchView bv, const float* __restrict__ pos_w, const float* __restrict__ pos_b,
    const float* __restrict__ coords, const uint8_t* __restrict__ src,
    const int* __restrict__ e_idx, float* __restrict__ feat) {
  const int r = blockIdx.x;
  const int b = bv.res_prot[r];
  const int off = bv.prot_res_off[b];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  const int i = r - off;
  // positional block: K*16 values; padding rows zeroed.
  for (int e = threadIdx.x; e < kK * 16; e += blockDim.x) {
    const int k = e >> 4, d = e & 15;
    float v = 0.0f;
    const int j = k < K ? e_idx[(int64_t)r * kK + k] : -1;
    if (j >= 0 && j < L) {
      int o = i - j;
      o = o < -32 ? -32 : (o > 32 ? 32 : o);
      v = pos_w[d * kPosClasses + o + 32] + pos_b[d];
    }
    feat[((int64_t)r * kK + k) * kEdgeIn + d] = v;
  }
  for (int e = threadIdx.x; e < kK * kPairs; e += blockDim.x) {
    const int k = e / kPairs, p = e % kPairs;
    float* out = feat + ((int64_t)r * kK + k) * kEdgeIn + 16 + p * 16;
    const int j = k < K ? e_idx[(int64_t)r * kK + k] : -1;
    const int a = c_pairs[p][0], bb = c_pairs[p][1];
    if (j < 0 || j >= L || !src[(int64_t)r * 5 + a] || !src[(int64_t)(off + j) * 5 + bb]) {
#pragma unroll
      for (int f = 0; f < 16; ++f) out[f] = 0.0f;
      continue;
    }
    const float dist = pair_distance(coords + ((int64_t)r * 5 + a) * 3,
                                     coords + ((int64_t)(off + j) * 5 + bb) * 3);
#pragma unroll
    for (int f = 0; f < 16; ++f) out[f] = rbf_value(dist, f);
  }
}

// ---------------------------------------------------------------------------
// Row LayerNorm family (one warp per 128-wide row).
// ---------------------------------------------------------------------------
__global__ void ln_rows_kernel(int64_t rows, const float* __restrict__ x,
                               const float* __restrict__ y,
                               const float* __restrict__ ybias,
                               const float* __restrict__ g,
                               const float* __restrict__ b,
                               const float* __restrict__ row_mask,
                               const int* __restrict__ row_to_mask,
                               float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[4];
  const int c = lane * 4;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float t = x[row * kH + c + u];
    if (y) t += y[row * kH + c + u] + (ybias ? ybias[c + u] : 0.0f);
    v[u] = t;
  }
  warp_layer_norm128(v, g, b, lane);
  float m = 1.0f;
  if (row_mask) m = row_mask[row_to_mask ? row_to_mask[row] : row];
#pragma unroll
  for (int u = 0; u < 4; ++u) out[row * kH + c + u] = (m == 1.0f) ? v[u] : v[u] * m;
}

// Encoder message / edge-update input: G1[r,k] = GELU(N_i + E_ik + N_j) with
// N = [W1a h + b1 | W1c h] (NAC, [R,256]) and E = W1b h_E (EB, [R*48,128]):
// the concatenated [h_i | e_ij | h_j] x W1^T of proteinmpnn_encoder_scalar.cpp:
// 169-213 split by input block.
__global__ void enc_msg_in_kernel(BatchView bv, const float* __restrict__ NAC,
                                  const float* __restrict__ EB,
                                  const int* __restrict__ e_idx,
                                  float* __restrict__ G1) {
  const int64_t s = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= (int64_t)bv.total_residues * kK) return;
  const int r = (int)(s / kK), k = (int)(s % kK);
  const int b = bv.res_prot[r];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  const int j = k < K ? e_idx[s] : -1;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  if (j >= 0 && j < L) {
    const int rj = bv.prot_res_off[b] + j;
    const float4 na = reinterpret_cast<const float4*>(NAC + (int64_t)r * 256)[lane];
    const float4 nc = reinterpret_cast<const float4*>(NAC + (int64_t)rj * 256 + 128)[lane];
    const float4 eb = reinterpret_cast<const float4*>(EB + s * kH)[lane];
    o.x = gelu_as(na.x + eb.x + nc.x);
    o.y = gelu_as(na.y + eb.y + nc.y);
    o.z = gelu_as(na.z + eb.z + nc.z);
    o.w = gelu_as(na.w + eb.w + nc.w);
  }
  reinterpret_cast<float4*>(G1 + s * kH)[lane] = o;
}

// S_i = sum_k m_i m_j G2[i,k], cnt_i = sum_k m_i m_j over valid neighbours
// (aggregate_messages_and_update_nodes, proteinmpnn_encoder_scalar.cpp:215-243;
// W3 and its bias are applied after the sum: sum_k a_k (W3 g_k + b3) =
// W3 (sum_k a_k g_k) + (sum_k a_k) b3).
__global__ void enc_aggregate_kernel(BatchView bv, const float* __restrict__ G2,
                                     const int* __restrict__ e_idx,
                                     const float* __restrict__ mask,
                                     float* __restrict__ S, float* __restrict__ cnt) {
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= bv.total_residues) return;
  const int b = bv.res_prot[r];
  const int off = bv.prot_res_off[b];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float c = 0.0f;
  for (int k = 0; k < K; ++k) {
    const int j = e_idx[(int64_t)r * kK + k];
    if (j < 0 || j >= L) continue;
    const float a = mask[r] * mask[off + j];
    if (a == 0.0f) continue;
    const float4 g = reinterpret_cast<const float4*>(G2 + ((int64_t)r * kK + k) * kH)[lane];
    acc.x += a * g.x;
    acc.y += a * g.y;
    acc.z += a * g.z;
    acc.w += a * g.w;
    c += a;
  }
  reinterpret_cast<float4*>(S + (int64_t)r * kH)[lane] = acc;
  if (lane == 0) cnt[r] = c;
}

// out = LN(h + (T3 + cnt * b3) / 30).
__global__ void node_update_kernel(int64_t rows, const float* __restrict__ T3,
                                   const float* __restrict__ cnt,
                                   const float* __restrict__ b3,
                                   const float* __restrict__ h,
                                   const float* __restrict__ g,
                                   const float* __restrict__ bb,
                                   float* __restrict__ out) {
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const float n = cnt[r];
  float v[4];
  const int c = lane * 4;
#pragma unroll
  for (int u = 0; u < 4; ++u)
    v[u] = h[r * kH + c + u] + (T3[r * kH + c + u] + n * b3[c + u]) * (1.0f / kMessageScale);
  warp_layer_norm128(v, g, bb, lane);
#pragma unroll
  for (int u = 0; u < 4; ++u) out[r * kH + c + u] = v[u];
}

// h_E[s] = LN3(h_E[s] + U3[s]) on valid slots (proteinmpnn_encoder_scalar.cpp:
// 312-320).
__global__ void edge_ln_update_kernel(BatchView bv, const float* __restrict__ U3,
                                      const int* __restrict__ e_idx,
                                      const float* __restrict__ g,
                                      const float* __restrict__ bb,
                                      float* __restrict__ h_e) {
  const int64_t s = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= (int64_t)bv.total_residues * kK) return;
  const int r = (int)(s / kK), k = (int)(s % kK);
  const int b = bv.res_prot[r];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  if (k >= K) return;
  const int j = e_idx[s];
  if (j < 0 || j >= L) return;
  float v[4];
  const int c = lane * 4;
#pragma unroll
  for (int u = 0; u < 4; ++u) v[u] = U3[s * kH + c + u] + h_e[s * kH + c + u];
  warp_layer_norm128(v, g, bb, lane);
#pragma unroll
  for (int u = 0; u < 4; ++u) h_e[s * kH + c + u] = v[u];
}

__global__ void gather_rows_kernel(int64_t rows, const int* __restrict__ row_res,
                                   const float* __restrict__ src,
                                   float* __restrict__ dst) {
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= rows) return;
  reinterpret_cast<float4*>(dst + q * kH)[lane] =
      reinterpret_cast<const float4*>(src + (int64_t)row_res[q] * kH)[lane];
}

// Teacher-forced decoder slot input for layer l (inverse_fold_scalar.cpp:
// 575-644 with the W1 split): with AP = [W1a h^l + b1 | W1d h^l] per row,
//   G1[q,k] = GELU(A_q + W1b h_E[t,k] + (bw ? W1c W_s[tok_j] + W1d h^l_j
//                                              : W1d h^enc_j)),
// bw = pos(j) < pos(t): neighbour j already decoded in this row's order.
__global__ void tf_slot_in_kernel(BatchView bv, TfRows tr, int layer,
                                  const float* __restrict__ AP,
                                  const float* __restrict__ PE,
                                  const float* __restrict__ PVenc,
                                  const float* __restrict__ Stab,
                                  const int* __restrict__ e_idx,
                                  float* __restrict__ G1) {
  const int64_t s = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (s >= tr.rows * kK) return;
  const int64_t q = s / kK;
  const int k = (int)(s % kK);
  const int r = tr.row_res[q];
  const int b = tr.row_prot[q];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  const int j = k < K ? e_idx[(int64_t)r * kK + k] : -1;
  if (j >= 0 && j < L) {
    const int rj = bv.prot_res_off[b] + j;
    const int64_t qj = tr.row_seqbase[q] + j;
    const bool bw = tr.pos[qj] < tr.pos[q];
    const float4 a = reinterpret_cast<const float4*>(AP + q * 256)[lane];
    const float4 pe = reinterpret_cast<const float4*>(PE + ((int64_t)r * kK + k) * kH)[lane];
    float4 v;
    if (bw) {
      const float4 st = reinterpret_cast<const float4*>(Stab + tr.tokens[qj] * kH)[lane];
      const float4 pv = reinterpret_cast<const float4*>(AP + qj * 256 + 128)[lane];
      v = make_float4(st.x + pv.x, st.y + pv.y, st.z + pv.z, st.w + pv.w);
    } else {
      v = reinterpret_cast<const float4*>(PVenc + (int64_t)rj * kH)[lane];
    }
    o.x = gelu_as(a.x + pe.x + v.x);
    o.y = gelu_as(a.y + pe.y + v.y);
    o.z = gelu_as(a.z + pe.z + v.z);
    o.w = gelu_as(a.w + pe.w + v.w);
  }
  reinterpret_cast<float4*>(G1 + s * kH)[lane] = o;
  (void)layer;
}

__global__ void row_slot_sum_kernel(BatchView bv, TfRows tr,
                                    const float* __restrict__ G2,
                                    float* __restrict__ S,
                                    float* __restrict__ kcount) {
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= tr.rows) return;
  const int L = bv.prot_len[tr.row_prot[q]];
  const int K = L < kK ? L : kK;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < K; ++k) {
    const float4 g = reinterpret_cast<const float4*>(G2 + (q * kK + k) * kH)[lane];
    acc.x += g.x;
    acc.y += g.y;
    acc.z += g.z;
    acc.w += g.w;
  }
  reinterpret_cast<float4*>(S + q * kH)[lane] = acc;
  if (lane == 0) kcount[q] = (float)K;
}

// Unscaled log-softmax of 21 logits per row (log_softmax_scalar.cpp:8-37).
__global__ void log_softmax_rows_kernel(int64_t rows, const float* __restrict__ z,
                                        float* __restrict__ out) {
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= rows) return;
  const float v = lane < kV ? z[q * kV + lane] : -INFINITY;
  const float mx = warp_max(v);
  const float e = lane < kV ? expf(v - mx) : 0.0f;
  const float ls = logf(warp_sum(e));
  if (lane < kV) out[q * kV + lane] = (v - mx) - ls;
}

// score = -mean over active residues of log_probs[t, token_t] (double
// accumulation; inverse_fold_scalar.cpp:471-493).  One warp per sequence.
__global__ void scores_kernel(BatchView bv, const int* __restrict__ tokens,
                              const float* __restrict__ lp,
                              const float* __restrict__ mask,
                              float* __restrict__ scores,
                              const float* __restrict__ lp_tok) {
  const int sq = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (sq >= bv.num_sequences) return;
  const int b = bv.seq_prot[sq];
  const int off = bv.prot_res_off[b];
  const int L = bv.prot_len[b];
  const int64_t q0 = bv.seq_row_off[sq];
  double loss = 0.0, cnt = 0.0;
  for (int t = lane; t < L; t += 32) {
    const float m = mask[off + t];
    const int tok = tokens[q0 + t];
    if (m == 0.0f || tok < 0 || tok >= kV) continue;
    loss -= (double)(lp_tok ? lp_tok[q0 + t] : lp[(q0 + t) * kV + tok]);
    cnt += (double)m;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    loss += __shfl_xor_sync(0xffffffffu, loss, o);
    cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  }
  if (lane == 0) scores[sq] = cnt > 0.0 ? (float)(loss / cnt) : 0.0f;
}

// ---------------------------------------------------------------------------
// Fused persistent autoregressive decode, fp32 SIMT (parity mode).
//
// One CTA owns up to kG sequences of one protein and walks all L decode
// positions.  At position p each sequence decodes its residue t = order[p]
// through the three DecLayers and the sampler (inverse_fold_scalar.cpp:
// 801-879), restated with the W1 split
//   W1 [h_t | h_E | h_S_j | h_j] = W1a h_t + W1b h_E + W1c W_s[tok_j] + W1d h_j
// so the per-slot work is a gather-add of precomputed 128-vectors, the W2
// contraction is the only per-slot GEMM, and W3 moves after the slot sum.
// W1d h^l_t (l = 1, 2) is stored per sequence when t is decoded so later
// positions gather it instead of recomputing it.
// ---------------------------------------------------------------------------
constexpr int kG = 4;            // sequences per CTA
constexpr int kArThreads = 256;

struct ArSmem {
  float h[kG][kH];
  float a[kG][kH];
  float s2[kG][kH];
  float hn[kG][kH];
  float f[kG][kFfn];
  float logits[kG][32];
  float g1[kG * kK][kH];
  int t[kG];
  float m[kG];
  int64_t qrow[kG];
  unsigned long long rng[kG];
  float temp[kG];
};

__device__ __forceinline__ float dot128_T(const float* __restrict__ x,
                                          const float* __restrict__ WT, int ldw,
                                          int o) {
  float acc = 0.0f;
#pragma unroll 8
  for (int i = 0; i < kH; ++i) acc = fmaf(x[i], WT[i * ldw + o], acc);
  return acc;
}

__device__ __forceinline__ unsigned long long splitmix64_next(unsigned long long& s) {
  unsigned long long z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Temperature softmax, emitted log-probs and the multinomial / greedy draw for
// one row, serial over the 21 logits in the reference's order
// (sampler_scalar.cpp:27-131).  Returns the token.
__device__ int sample_row(const float* z, float temperature, unsigned long long& rng,
                          float* lp_out) {
  const bool greedy = !(temperature > 0.0f);
  const float T = (temperature > 0.0f && isfinite(temperature)) ? temperature : 1.0f;
  float zz[kV];
  float mx = -INFINITY;
  for (int v = 0; v < kV; ++v) {
    zz[v] = z[v] / T;
    mx = fmaxf(mx, zz[v]);
  }
  float prob[kV];
  float sum = 0.0f;
  for (int v = 0; v < kV; ++v) {
    prob[v] = expf(zz[v] - mx);
    sum += prob[v];
  }
  const float ls = logf(sum), inv = 1.0f / sum;
  for (int v = 0; v < kV; ++v) {
    prob[v] *= inv;
    lp_out[v] = (zz[v] - mx) - ls;
  }
  if (greedy) {
    int best = 0;
    for (int v = 1; v < kV; ++v)
      if (zz[v] > zz[best]) best = v;
    return best;
  }
  const double u = (double)(splitmix64_next(rng) >> 11) * (1.0 / 9007199254740992.0);
  double cum = 0.0;
  for (int v = 0; v < kV; ++v) {
    cum += (double)prob[v];
    if (u < cum) return v;
  }
  return kV - 1;
}

__global__ void __launch_bounds__(kArThreads) ar_decode_f32_kernel(
    BatchView bv, F32Weights w, DecoderTables dt, ArArgs a, unsigned int* err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  ArSmem& S = *reinterpret_cast<ArSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int g = blockIdx.x;
  const int seq0 = a.group_seq0[g];
  const int n = a.group_count[g];
  const int b = bv.seq_prot[seq0];
  const int off = bv.prot_res_off[b];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;

  if (tid < kG) {
    const bool live = tid < n;
    S.qrow[tid] = live ? bv.seq_row_off[seq0 + tid] : 0;
    S.rng[tid] = live ? a.seq_seed[seq0 + tid] : 0ull;
    S.temp[tid] = live ? a.seq_temp[seq0 + tid] : 1.0f;
  }
  __syncthreads();
  for (int s = 0; s < n; ++s)
    for (int p = tid; p < L; p += kArThreads) {
      const int t = a.orders[S.qrow[s] + p];
      if (t < 0 || t >= L) {
        set_err(err, kErrBadIndex);
        continue;
      }
      a.pos[S.qrow[s] + t] = p;
    }
  __syncthreads();

  for (int p = 0; p < L; ++p) {
    if (tid < kG) {
      int t = 0;
      float m = 0.0f;
      if (tid < n) {
        t = a.orders[S.qrow[tid] + p];
        t = (t < 0 || t >= L) ? 0 : t;
        m = a.mask[off + t];
      }
      S.t[tid] = t;
      S.m[tid] = m;
    }
    __syncthreads();
    for (int e = tid; e < kG * kH; e += kArThreads) {
      const int s = e / kH, c = e % kH;
      S.h[s][c] = (s < n) ? a.h_enc[(int64_t)(off + S.t[s]) * kH + c] : 0.0f;
    }
    __syncthreads();

    for (int l = 0; l < 3; ++l) {
      const F32Weights::Dec& D = w.dec[l];
      // (1) node term A_t = W1a h_t + b1
      for (int e = tid; e < kG * kH; e += kArThreads) {
        const int s = e / kH, o = e % kH;
        float v = 0.0f;
        if (s < n) {
          if (l == 0) v = dt.Aenc0[(int64_t)(off + S.t[s]) * kH + o];
          else v = D.b1[o] + dot128_T(S.h[s], D.W1aT, kH, o);
        }
        S.a[s][o] = v;
      }
      __syncthreads();
      // (2) per-slot gather-add + GELU
      const float* PE = dt.PE[l];
      const float* PVenc = dt.PVenc[l];
      const float* PV = l > 0 ? a.PV + (int64_t)(l - 1) * a.total_rows * kH : nullptr;
      for (int e = tid; e < n * K * 32; e += kArThreads) {
        const int row = e >> 5, c4 = e & 31;
        const int s = row / K, k = row % K;
        const int t = S.t[s];
        const int64_t rt = off + t;
        int j = a.e_idx[rt * kK + k];
        if (j < 0 || j >= L) {
          set_err(err, kErrBadIndex);
          j = t;
        }
        const int64_t qj = S.qrow[s] + j;
        const bool bw = a.pos[qj] < p;
        const float4 av = reinterpret_cast<const float4*>(S.a[s])[c4];
        const float4 pe = reinterpret_cast<const float4*>(PE + (rt * kK + k) * kH)[c4];
        float4 vv;
        if (bw && l > 0) vv = reinterpret_cast<const float4*>(PV + qj * kH)[c4];
        else vv = reinterpret_cast<const float4*>(PVenc + (int64_t)(off + j) * kH)[c4];
        if (bw) {
          const float4 st = reinterpret_cast<const float4*>(D.Stab + a.tokens[qj] * kH)[c4];
          vv.x += st.x; vv.y += st.y; vv.z += st.z; vv.w += st.w;
        }
        float4 o;
        o.x = gelu_as(av.x + pe.x + vv.x);
        o.y = gelu_as(av.y + pe.y + vv.y);
        o.z = gelu_as(av.z + pe.z + vv.z);
        o.w = gelu_as(av.w + pe.w + vv.w);
        reinterpret_cast<float4*>(S.g1[s * kK + k])[c4] = o;
      }
      __syncthreads();
      // (3) W2 contraction, GELU and slot sum
      {
        const int o = tid % kH;
        const int half = tid / kH;
        for (int s = half; s < n; s += 2) {
          float total = 0.0f;
          for (int kb = 0; kb < K; kb += 8) {
            float acc[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[u] = D.b2[o];
            const float* g1base = S.g1[s * kK + kb];
            for (int i = 0; i < kH; ++i) {
              const float wv = D.W2T[i * kH + o];
#pragma unroll
              for (int u = 0; u < 8; ++u) acc[u] = fmaf(g1base[u * kH + i], wv, acc[u]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
              if (kb + u < K) total += gelu_as(acc[u]);
          }
          S.s2[s][o] = total;
        }
      }
      __syncthreads();
      // (4) W3 after the sum, residual + LayerNorm 1
      for (int e = tid; e < kG * kH; e += kArThreads) {
        const int s = e / kH, o = e % kH;
        float v = 0.0f;
        if (s < n) {
          const float d = (dot128_T(S.s2[s], D.W3T, kH, o) + (float)K * D.b3[o]) *
                          (1.0f / kMessageScale);
          v = S.h[s][o] + d;
        }
        S.hn[s][o] = v;
      }
      __syncthreads();
      {
        const int wp = tid >> 5, lane = tid & 31;
        if (wp < n) {
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = S.hn[wp][lane * 4 + u];
          warp_layer_norm128(v, D.n1w, D.n1b, lane);
#pragma unroll
          for (int u = 0; u < 4; ++u) S.hn[wp][lane * 4 + u] = v[u];
        }
      }
      __syncthreads();
      // (5) FFN 128 -> 512 -> 128, residual + LayerNorm 2, residue mask
      for (int e = tid; e < kG * kFfn; e += kArThreads) {
        const int s = e / kFfn, u = e % kFfn;
        float v = 0.0f;
        if (s < n) v = gelu_as(D.bin[u] + dot128_T(S.hn[s], D.WinT, kFfn, u));
        S.f[s][u] = v;
      }
      __syncthreads();
      for (int e = tid; e < kG * kH; e += kArThreads) {
        const int s = e / kH, o = e % kH;
        float v = 0.0f;
        if (s < n) {
          float acc = D.bout[o];
#pragma unroll 8
          for (int u = 0; u < kFfn; ++u) acc = fmaf(S.f[s][u], D.WoutT[u * kH + o], acc);
          v = S.hn[s][o] + acc;
        }
        S.a[s][o] = v;
      }
      __syncthreads();
      {
        const int wp = tid >> 5, lane = tid & 31;
        if (wp < n) {
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = S.a[wp][lane * 4 + u];
          warp_layer_norm128(v, D.n2w, D.n2b, lane);
          const float m = S.m[wp];
#pragma unroll
          for (int u = 0; u < 4; ++u) S.h[wp][lane * 4 + u] = (m == 1.0f) ? v[u] : v[u] * m;
        }
      }
      __syncthreads();
      // (6) W1d_{l+1} h^{l+1}_t for later neighbours of t
      if (l < 2) {
        const F32Weights::Dec& Dn = w.dec[l + 1];
        float* PVn = a.PV + (int64_t)l * a.total_rows * kH;
        for (int e = tid; e < kG * kH; e += kArThreads) {
          const int s = e / kH, o = e % kH;
          if (s < n && S.m[s] != 0.0f)
            PVn[(S.qrow[s] + S.t[s]) * kH + o] = dot128_T(S.h[s], Dn.W1dT, kH, o);
        }
      }
    }
    // logits and sampling
    for (int e = tid; e < kG * 32; e += kArThreads) {
      const int s = e / 32, v = e % 32;
      float z = 0.0f;
      if (s < n && v < kV) z = w.head_b[v] + dot128_T(S.h[s], w.headT, kV, v);
      S.logits[s][v] = z;
    }
    __syncthreads();
    if (tid < n) {
      const int s = tid;
      const int t = S.t[s];
      const int64_t q = S.qrow[s] + t;
      float* lp = a.log_probs + q * kV;
      int tok;
      if (S.m[s] == 0.0f) {
        tok = kV - 1;
        for (int v = 0; v < kV; ++v) lp[v] = 0.0f;
      } else {
        float row[kV];
        tok = sample_row(S.logits[s], S.temp[s], S.rng[s], row);
        for (int v = 0; v < kV; ++v) lp[v] = row[v];
      }
      a.tokens[q] = tok;
    }
    __syncthreads();
  }
}

inline unsigned grid_rows(int64_t rows, int rows_per_block) {
  return (unsigned)((rows + rows_per_block - 1) / rows_per_block);
}

}  // namespace

void gemm_f32(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
              const float* B, int ldb, const float* bias, int act, float* C,
              int ldc) {
  if (M <= 0) return;
  if (gemm_f32x2_fits(N, K, A, lda, B, ldb, C, ldc)) {
    gemm_f32x2(st, M, N, K, A, lda, B, ldb, bias, act, C, ldc, false);
    return;
  }
  dim3 grid((unsigned)((M + 63) / 64), (N + 63) / 64);
  if (act == 1)
    gemm_f32_kernel<1><<<grid, 256, 0, st>>>(M, N, K, A, lda, B, ldb, bias, C, ldc);
  else
    gemm_f32_kernel<0><<<grid, 256, 0, st>>>(M, N, K, A, lda, B, ldb, bias, C, ldc);
}

bool gemm_f32x2_fits(int N, int K, const void* A, int lda, const void* B, int ldb,
                     const void* C, int ldc) {
  auto al16 = [](const void* p) { return ((uintptr_t)p & 15u) == 0; };
  return N > 0 && N % kG2Tile == 0 && K > 0 && K % kG2K == 0 && lda % 4 == 0 &&
         ldb % 4 == 0 && ldc % 8 == 0 && al16(A) && al16(B) && al16(C);
}

void gemm_f32x2(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
                const float* B, int ldb, const float* bias, int act, void* C, int ldc,
                bool out_f16) {
  if (M <= 0) return;
  ensure_dynamic_smem((const void*)gemm_f32x2_kernel<0, false>, (int)kG2Smem);
  ensure_dynamic_smem((const void*)gemm_f32x2_kernel<1, false>, (int)kG2Smem);
  ensure_dynamic_smem((const void*)gemm_f32x2_kernel<0, true>, (int)kG2Smem);
  ensure_dynamic_smem((const void*)gemm_f32x2_kernel<1, true>, (int)kG2Smem);
  const dim3 grid((unsigned)((M + kG2Tile - 1) / kG2Tile), N / kG2Tile);
  if (out_f16) {
    if (act == 1)
      gemm_f32x2_kernel<1, true><<<grid, 256, kG2Smem, st>>>(M, K, A, lda, B, ldb, bias, C, ldc);
    else
      gemm_f32x2_kernel<0, true><<<grid, 256, kG2Smem, st>>>(M, K, A, lda, B, ldb, bias, C, ldc);
  } else {
    if (act == 1)
      gemm_f32x2_kernel<1, false><<<grid, 256, kG2Smem, st>>>(M, K, A, lda, B, ldb, bias, C, ldc);
    else
      gemm_f32x2_kernel<0, false><<<grid, 256, kG2Smem, st>>>(M, K, A, lda, B, ldb, bias, C, ldc);
  }
}

void launch_knn(cudaStream_t st, const BatchView& bv, const float* coords,
                const uint8_t* sources, int* e_idx, float* d2, float* mask,
                unsigned int* err, int max_len) {
  if (bv.total_residues <= 0) return;
  // One shared-memory key per candidate of the query's protein.
  const size_t smem = (size_t)max_len * sizeof(unsigned long long);
  ensure_dynamic_smem((const void*)knn_kernel, kMaxResidues * (int)sizeof(unsigned long long));
  knn_kernel<<<bv.total_residues, 256, smem, st>>>(bv, coords, sources, e_idx, d2,
                                                   mask, err);
}

void launch_edge_features(cudaStream_t st, const BatchView& bv, const F32Weights& w,
                          const float* coords, const uint8_t* sources,
                          const int* e_idx, float* feat) {
  if (bv.total_residues <= 0) return;
  edge_features_kernel<<<bv.total_residues, 256, 0, st>>>(bv, w.pos_w, w.pos_b, coords,
                                                          sources, e_idx, feat);
}

void launch_ln_rows(cudaStream_t st, int64_t rows, const float* x, const float* y,
                    const float* ybias, const float* g, const float* b,
                    const float* row_mask, const int* row_to_mask, float* out) {
  if (rows <= 0) return;
  ln_rows_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(rows, x, y, ybias, g, b, row_mask,
                                                     row_to_mask, out);
}

void launch_enc_msg_in(cudaStream_t st, const BatchView& bv, const float* NAC,
                       const float* EB, const int* e_idx, float* G1) {
  const int64_t slots = (int64_t)bv.total_residues * kK;
  if (slots <= 0) return;
  enc_msg_in_kernel<<<grid_rows(slots, 8), 256, 0, st>>>(bv, NAC, EB, e_idx, G1);
}

void launch_enc_aggregate(cudaStream_t st, const BatchView& bv, const float* G2,
                          const int* e_idx, const float* mask, float* S, float* cnt) {
  if (bv.total_residues <= 0) return;
  enc_aggregate_kernel<<<grid_rows(bv.total_residues, 8), 256, 0, st>>>(bv, G2, e_idx,
                                                                        mask, S, cnt);
}

void launch_enc_node_update(cudaStream_t st, const BatchView& bv, const float* T3,
                            const float* cnt, const float* b3, const float* h,
                            const float* g, const float* b, float* out) {
  if (bv.total_residues <= 0) return;
  node_update_kernel<<<grid_rows(bv.total_residues, 8), 256, 0, st>>>(
      bv.total_residues, T3, cnt, b3, h, g, b, out);
}

void launch_dec_node_update(cudaStream_t st, int64_t rows, const float* T3,
                            const float* kcount, const float* b3, const float* h,
                            const float* g, const float* b, float* out) {
  if (rows <= 0) return;
  node_update_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(rows, T3, kcount, b3, h, g, b,
                                                         out);
}

void launch_edge_ln_update(cudaStream_t st, const BatchView& bv, const float* U3,
                           const int* e_idx, const float* g, const float* b,
                           float* h_e) {
  const int64_t slots = (int64_t)bv.total_residues * kK;
  if (slots <= 0) return;
  edge_ln_update_kernel<<<grid_rows(slots, 8), 256, 0, st>>>(bv, U3, e_idx, g, b, h_e);
}

void launch_gather_rows(cudaStream_t st, int64_t rows, const int* row_res,
                        const float* src, float* dst) {
  if (rows <= 0) return;
  gather_rows_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(rows, row_res, src, dst);
}

void launch_tf_slot_in(cudaStream_t st, const BatchView& bv, const TfRows& tr,
                       int layer, const float* AP, const DecoderTables& dt,
                       const float* Stab, const int* e_idx, float* G1) {
  const int64_t slots = tr.rows * kK;
  if (slots <= 0) return;
  tf_slot_in_kernel<<<grid_rows(slots, 8), 256, 0, st>>>(
      bv, tr, layer, AP, dt.PE[layer], dt.PVenc[layer], Stab, e_idx, G1);
}

void launch_row_slot_sum(cudaStream_t st, const BatchView& bv, const TfRows& tr,
                         const float* G2, float* S, float* kcount) {
  if (tr.rows <= 0) return;
  row_slot_sum_kernel<<<grid_rows(tr.rows, 8), 256, 0, st>>>(bv, tr, G2, S, kcount);
}

void launch_log_softmax_rows(cudaStream_t st, int64_t rows, const float* logits,
                             float* out) {
  if (rows <= 0) return;
  log_softmax_rows_kernel<<<grid_rows(rows, 8), 256, 0, st>>>(rows, logits, out);
}

void launch_scores(cudaStream_t st, const BatchView& bv, const int* tokens,
                   const float* log_probs, const float* mask, float* scores,
                   const float* lp_tok) {
  if (bv.num_sequences <= 0) return;
  scores_kernel<<<grid_rows(bv.num_sequences, 8), 256, 0, st>>>(bv, tokens, log_probs,
                                                               mask, scores, lp_tok);
}

void launch_ar_decode_f32(cudaStream_t st, const BatchView& bv, const F32Weights& w,
                          const DecoderTables& dt, const ArArgs& a, unsigned int* err) {
  if (a.num_groups <= 0) return;
  const size_t smem = sizeof(ArSmem);
  ensure_dynamic_smem((const void*)ar_decode_f32_kernel, (int)smem);
  ar_decode_f32_kernel<<<a.num_groups, kArThreads, smem, st>>>(bv, w, dt, a, err);
}

int ar_f32_group_size() { return kG; }

}  // namespace hkb
