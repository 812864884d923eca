// Teacher-forced scoring on tcgen05 tensor cores (fp16 operands, fp32
// accumulation, LayerNorm and softmax): the parallel causally masked decoder
// pass of run_teacher_forced_decoder (inverse_fold_scalar.cpp:575-663) over
// every (sequence, residue) row at once.  Each of the three decoder layers is
// two persistent kernels:
//
//   tf_slot_tc   one residue t per work item, all of its protein's sequences
//     D1 = W1b h_E[t]                       M = 128 features, N = 48 slots
//     G  = GELU(D1 + A_row + V_slot)        per row (sequence) and slot k
//        V_slot = PV_l[s, j] + W1c W_s[tok_j]   if pos_s(j) < pos_s(t)
//               = W1d h_enc[j]                  otherwise
//     D2 = W2 G                             N = 48 slots x up to 2 rows
//     S_row = sum_{k < K} GELU(D2 + b2)
//   The W1b h_E term is computed once per residue and shared by its rows.
//
//   tf_node_tc   128 rows per tile (rows on TMEM lanes, weights as B)
//     h1 = LN1(h + (W3 S + K b3) / 30)
//     h' = LN2(h1 + W_out GELU(W_in h1 + b_in) + b_out) * m_t
//     (W_in as fp16 value + fp16 remainder), then the next layer's node
//     terms A = W1a h' + b1 (fp32) and
//     PV = W1d h' (fp16), or, after the last layer, the logits and their
//     unscaled log-softmax (log_softmax_scalar.cpp:8-37).
//   Weight tiles stream through a 3-slot shared-memory ring by bulk copies.
//
// The split W1 . [h_t | h_E | W_s tok_j | h_j] = W1a h_t + W1b h_E + W1c W_s
// tok_j + W1d h_j and W3 after the slot sum are exact in real arithmetic
// (the same restatement as the autoregressive kernel).  Every wait is bounded.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace hkb {
namespace {

using namespace tc;

constexpr int kTfThreads = 512;
constexpr uint32_t kW128 = 128 * 128 * 2;

__device__ __forceinline__ uint32_t idesc_h(int M, int N) {
  return idesc_bf16(M, N) & ~((7u << 7) | (7u << 10));
}

// ---------------------------------------------------------------------------
// Slot kernel
// ---------------------------------------------------------------------------
// Two ping-pong groups of 8 warps.  Per work item (one residue t) the CTA
// forms D1 = W1b h_E[t] once; then group g takes the sub-tiles g, g+2, ... of
// two sequences (96 slots) each: it stages the slots' gather addresses,
// builds its G operand, issues its W2 MMA into its own TMEM columns and sums
// the slots, so that one group's MMA wait and slot sum overlap the other
// group's gathers and GELUs.  A thread owns one feature (f = TMEM lane) of one
// row of its group's sub-tile.
constexpr int kSubRows = 2;                        // rows per W2 MMA and group
constexpr int kSubN = kSubRows * kK;               // 96 slots
constexpr uint32_t kSOffW1b = 0;
constexpr uint32_t kSOffW2 = kW128;
constexpr uint32_t kSOffE = 2 * kW128;             // 2 h_E tiles of 48 rows
constexpr uint32_t kETileBytes = kK * 256;         // 12 KiB
constexpr uint32_t kSOffG = kSOffE + 2 * kETileBytes;
constexpr uint32_t kGBytes = kSubN * 256;          // 24 KiB per group
constexpr uint32_t kSOffStab = kSOffG + 2 * kGBytes;   // fp32 [22,128] (row 21 zero)
constexpr uint32_t kSOffSrc = kSOffStab + (kV + 1) * kH * 4; // per group, 2 buffers: [96] row pointers
constexpr uint32_t kSOffSt = kSOffSrc + 4 * kSubN * 8; // per group, 2 buffers: [96] Stab row
constexpr uint32_t kSOffJ = kSOffSt + 4 * kSubN * 4;   // int [48] local neighbour
constexpr uint32_t kSOffD1 = kSOffJ + kK * 4;          // fp32 [48][128] D1, slot-major
constexpr uint32_t kSOffAS = kSOffD1 + kK * kH * 4;    // per group, 2 buffers: fp32 [2][128] A rows
constexpr uint32_t kSlotSmem = kSOffAS + 4 * kSubRows * kH * 4 + 1024;
static_assert(kSlotSmem <= 227 * 1024, "slot kernel shared memory");
constexpr uint32_t kTfColD2 = 64;                  // group g: columns 64 + 96 g
constexpr int kGroupThreadsTf = 256;

// The V row of a slot past K (its products are dropped by the slot sum).
__device__ __align__(16) const uint16_t g_zero_row[kH] = {};

__device__ __forceinline__ void load_etile(unsigned char* tile, const uint16_t* h_e, int64_t row0,
                                           int64_t row_end, int tid) {
  for (int c = tid; c < kK * 16; c += kTfThreads) {
    const int r = c >> 4, k8 = c & 15;
    const int64_t gr = row0 + r;
    const bool ok = gr < row_end;
    cp_async16(tile + sw128_offset(r, k8 * 8, kK), h_e + (ok ? gr : 0) * kH + k8 * 8, ok);
  }
}

__global__ void __launch_bounds__(kTfThreads, 1) tf_slot_tc_kernel(const __grid_constant__ TfSlotArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float* StabS = reinterpret_cast<float*>(sm + kSOffStab);
  int* SJ = reinterpret_cast<int*>(sm + kSOffJ);
  float* D1s = reinterpret_cast<float*>(sm + kSOffD1);
  __shared__ uint64_t bar_w, bar_d1, bar_d2[2];
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = warp >> 3, gtid = tid & (kGroupThreadsTf - 1);
  const int quad = warp & 3, rho = (warp >> 2) & 1;   // feature quadrant, row of the sub-tile
  const int f = quad * 32 + lane;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int R = p.bv.total_residues;
  const int64_t SL = (int64_t)R * kK;
  const int l = p.layer;
  const uint16_t** SRC0 = reinterpret_cast<const uint16_t**>(sm + kSOffSrc) + grp * 2 * kSubN;
  int* STR0 = reinterpret_cast<int*>(sm + kSOffSt) + grp * 2 * kSubN;
  unsigned char* G = sm + kSOffG + grp * kGBytes;
  float* AS0 = reinterpret_cast<float*>(sm + kSOffAS) + grp * 2 * kSubRows * kH;
  const uint16_t* PVl = l == 0 ? p.PVenc : p.PV;   // decoded neighbours' rows

  if (tid == 0) {
    mbar_init(&bar_w, 1);
    mbar_init(&bar_d1, 1);
    mbar_init(&bar_d2[0], 1);
    mbar_init(&bar_d2[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  for (int e = tid; e < (kV + 1) * kH; e += kTfThreads) StabS[e] = e < kV * kH ? p.Stab[e] : 0.0f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar_w, 2 * kW128);
    for (uint32_t o = 0; o < kW128; o += 16384u) {
      bulk_g2s(sm + kSOffW1b + o, p.W1b + o, 16384u, &bar_w);
      bulk_g2s(sm + kSOffW2 + o, p.W2 + o, 16384u, &bar_w);
    }
  }
  bool ok = mbar_wait(&bar_w, 0, p.err);
  uint32_t ph1 = 0, ph2 = 0;
  const float b2 = p.b2[f];
  const float2 b2p = make_float2(b2, b2);
  const float2 halfc = make_float2(0.5f, 0.5f);

  int r = blockIdx.x;
  if (r < R) load_etile(sm + kSOffE, p.h_e, (int64_t)r * kK, SL, tid);
  cp_async_commit();
  for (int it = 0; r < R; r += gridDim.x, ++it) {
    if (__syncthreads_or(!ok)) break;
    unsigned char* etile = sm + kSOffE + (it & 1) * kETileBytes;
    const int b = p.bv.res_prot[r];
    const int L = p.bv.prot_len[b];
    const int K = L < kK ? L : kK;
    const int off = p.bv.prot_res_off[b];
    const int t = r - off;
    const int seq0 = p.prot_seq0[b];
    const int nseq = p.prot_nseq[b];
    cp_async_wait_all();
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      mma_k128(tm, smem_u32(sm + kSOffW1b), smem_u32(etile), kK, idesc_h(128, kK), false);
      mma_commit(&bar_d1);
    }
    if (tid < kK) {
      int j = -1;
      if (tid < K) {
        j = p.e_idx[(int64_t)r * kK + tid];
        if (j < 0 || j >= L) {
          atomicOr(p.err, kErrBadIndex);
          j = -1;
        }
      }
      SJ[tid] = j;
    }
    if (!mbar_wait(&bar_d1, ph1, p.err)) ok = false;
    ph1 ^= 1;
    tc_fence_after();
    // the other h_E buffer was last read by the previous item's D1 MMA
    const int rn = r + gridDim.x;
    if (rn < R) load_etile(sm + kSOffE + ((it + 1) & 1) * kETileBytes, p.h_e, (int64_t)rn * kK, SL, tid);
    cp_async_commit();
    // D1 to shared memory, slot-major (D1s[k][f]): warp w reads its lane
    // quadrant's features for slots 12 (w / 4) .. 12 (w / 4) + 11
    {
      const int k0 = (warp >> 2) * 12;
      float v8[8], v4[4];
      tmem_ld8(tm + lane_base + (uint32_t)k0, v8);
      tmem_ld4(tm + lane_base + (uint32_t)(k0 + 8), v4);
#pragma unroll
      for (int i = 0; i < 8; ++i) D1s[(k0 + i) * kH + f] = v8[i];
#pragma unroll
      for (int i = 0; i < 4; ++i) D1s[(k0 + 8 + i) * kH + f] = v4[i];
    }
    tc_fence_before();
    __syncthreads();   // SJ and D1s visible; D1 read before the next item's MMA
    // Gather addresses of sub-tile `sub` into address buffer `ab` (threads
    // gtid < 96 of the group; their global loads overlap the group's MMA).
    // Per slot of sub-tile `sub`: the address of its V row (a decoded
    // neighbour's PV row or the neighbour's PVenc row; a zero row for a slot
    // past K, whose products the slot sum drops) and the offset of its W1c W_s
    // row in shared memory (row 21 is zero).  Threads gtid < 96 of the group;
    // their global loads overlap the group's MMA.
    auto stage = [&](int sub, int ab) {
      if (gtid < kSubN && sub * kSubRows < nseq) {
        const int s0 = sub * kSubRows;
        const int nrows = nseq - s0 < kSubRows ? nseq - s0 : kSubRows;
        const int rr = gtid / kK, k = gtid % kK;
        const uint16_t* src = g_zero_row;
        int st = kV * kH;
        const int j = SJ[k];
        if (rr < nrows && j >= 0) {
          const int64_t qs = p.bv.seq_row_off[seq0 + s0 + rr];
          const int64_t qj = qs + j;
          if (p.pos[qj] < p.pos[qs + t]) {   // decoded neighbour: its own row
            src = PVl + (l == 0 ? (int64_t)(off + j) : qj) * kH;
            st = p.tokens[qj] * kH;
          } else {                           // undecoded: the encoder row
            src = p.PVenc + (int64_t)(off + j) * kH;
          }
        }
        SRC0[ab * kSubN + gtid] = src;
        STR0[ab * kSubN + gtid] = st;
      } else if (gtid >= kSubN && gtid < kSubN + kSubRows * 32 && sub * kSubRows < nseq) {
        // the sub-tile's A rows (W1a h + b1 of each row, fp32) into AS[ab]
        const int s0 = sub * kSubRows;
        const int rr = (gtid - kSubN) >> 5, c4 = (gtid - kSubN) & 31;
        if (s0 + rr < nseq) {
          const float* arow = l == 0 ? p.Aenc0 + (int64_t)r * kH
                                     : p.A + (p.bv.seq_row_off[seq0 + s0 + rr] + t) * kH;
          reinterpret_cast<float4*>(AS0 + (ab * kSubRows + rr) * kH)[c4] =
              reinterpret_cast<const float4*>(arow)[c4];
        }
      }
    };
    stage(grp, 0);
    named_bar_sync(1 + grp, kGroupThreadsTf);
    int ab = 0;
    for (int sub = grp; sub * kSubRows < nseq; sub += 2, ab ^= 1) {
      const int s0 = sub * kSubRows;
      const int nrows = nseq - s0 < kSubRows ? nseq - s0 : kSubRows;
      const int N = nrows * kK;
      int64_t q = -1;   // the row this thread sums (feature f of row rho)
      if (rho < nrows) q = p.bv.seq_row_off[seq0 + s0 + rho] + t;
      // Build: thread (c8, r0) forms 8 consecutive features (8 c8 ..) of slot
      // rows r0, r0 + 16, ..., r0 + 80 of the sub-tile (row r = 48 rr + k):
      // 2 GELU(D1[k] + A_rr + V + W1c W_s[tok]) in fp32, one 16-byte fp16
      // store into the SW128 operand.  Slots past K get zeros (the slot sum
      // drops their products).
      {
        const int c8 = gtid & 15, r0 = gtid >> 4;
        const uint16_t* const* SRC = SRC0 + ab * kSubN;
        const int* STR = STR0 + ab * kSubN;
        const float* AS = AS0 + ab * kSubRows * kH;
#pragma unroll
        for (int i = 0; i < kSubN / 16; ++i) {
          const int rs = r0 + 16 * i;
          const int rr = rs / kK, k = rs % kK;
          if (rr >= nrows) continue;
          uint4 outv = make_uint4(0, 0, 0, 0);
          if (k < K) {
            const uint4 vr = *reinterpret_cast<const uint4*>(SRC[rs] + c8 * 8);
            const float4* d = reinterpret_cast<const float4*>(D1s + k * kH + c8 * 8);
            const float4* av = reinterpret_cast<const float4*>(AS + rr * kH + c8 * 8);
            const float4* sv = reinterpret_cast<const float4*>(StabS + STR[rs] + c8 * 8);
            const float4 d0 = d[0], d1v = d[1], a0 = av[0], a1 = av[1], t0 = sv[0], t1 = sv[1];
            const float dd[8] = {d0.x, d0.y, d0.z, d0.w, d1v.x, d1v.y, d1v.z, d1v.w};
            const float aa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float tt[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
            const uint32_t vw[4] = {vr.x, vr.y, vr.z, vr.w};
            uint32_t pk[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(&vw[u]));
              const float x0 = ((dd[2 * u] + aa[2 * u]) + vv.x) + tt[2 * u];
              const float x1 = ((dd[2 * u + 1] + aa[2 * u + 1]) + vv.y) + tt[2 * u + 1];
              // the operand holds 2 GELU(x); the epilogue halves D2 (exact)
              const float2 y = gelu2_tc_x2(make_float2(x0, x1));
              const __half2 h = __floats2half2_rn(y.x, y.y);
              pk[u] = *reinterpret_cast<const uint32_t*>(&h);
            }
            outv = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
          *reinterpret_cast<uint4*>(G + sw128_offset(rs, c8 * 8, N)) = outv;
        }
      }
      fence_async_smem();
      tc_fence_before();
      named_bar_sync(1 + grp, kGroupThreadsTf);
      if (gtid == 0) {
        tc_fence_after();
        if (ok) mma_k128(tm + kTfColD2 + grp * kSubN, smem_u32(sm + kSOffW2), smem_u32(G), N,
                         idesc_h(128, N), false);
        mma_commit(&bar_d2[grp]);
      }
      stage(sub + 2, ab ^ 1);   // the next sub-tile's addresses while the MMA runs
      if (!mbar_wait(&bar_d2[grp], ph2, p.err)) ok = false;
      ph2 ^= 1;
      tc_fence_after();
      if (rho < nrows) {
        float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
#pragma unroll
        for (int k0 = 0; k0 < kK; k0 += 16) {
          float v[16];
          tmem_ld16(tm + lane_base + kTfColD2 + (uint32_t)(grp * kSubN + rho * kK + k0), v);
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            float2 g = gelu2_tc_x2(__ffma2_rn(make_float2(v[k], v[k + 1]), halfc, b2p));
            if (k0 + k >= K) g.x = 0.0f;
            if (k0 + k + 1 >= K) g.y = 0.0f;
            acc[(k >> 1) & 1] = __fadd2_rn(acc[(k >> 1) & 1], g);
          }
        }
        p.S[q * kH + f] = 0.5f * ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y));
      }
      tc_fence_before();
      named_bar_sync(1 + grp, kGroupThreadsTf);   // G free, next addresses staged
    }
  }
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// Node kernel
// ---------------------------------------------------------------------------
constexpr int kRing = 3;
constexpr uint32_t kNOffRing = 0;                         // 3 x 32 KiB weight tiles
constexpr uint32_t kNOffA = kRing * kW128;                // A operand [128 rows x 128]
constexpr uint32_t kNOffF = kNOffA + kW128;               // 2 FFN operands
constexpr uint32_t kNOffRed = kNOffF + 2 * kW128;         // float [2][4][128]
constexpr uint32_t kNOffHead = kNOffRed + 2 * 4 * 128 * 4;   // fp32 [21][128]
constexpr uint32_t kNodeSmem = kNOffHead + kV * kH * 4 + 1024;
static_assert(kNodeSmem <= 227 * 1024, "node kernel shared memory");
// logits partials [21][4][128] fp32 reuse the FFN operand buffers
static_assert(kV * 4 * 128 * 4 <= 2 * kW128, "logit partials");

// TMEM columns
constexpr uint32_t kNColD = 0;      // W3 / W1a'
constexpr uint32_t kNColIn = 128;   // 2 x W_in chunk (the second reused by W1d')
constexpr uint32_t kNColOut = 384;  // W_out accumulator

struct Ring {
  int issued;
  int used;
  int total;
};

__device__ __forceinline__ void ring_issue(Ring& rg, unsigned char* sm, uint64_t* full,
                                           const TfNodeArgs& p, int per_tile) {
  while (rg.issued < rg.total && rg.issued < rg.used + kRing) {
    const int slot = rg.issued % kRing;
    const int tile = p.tile_ids[rg.issued % per_tile];
    mbar_arrive_expect_tx(&full[slot], kW128);
    bulk_g2s(sm + kNOffRing + slot * kW128, p.stream + (size_t)tile * kW128, kW128, &full[slot]);
    ++rg.issued;
  }
}

__device__ __forceinline__ uint32_t ring_wait(int j, unsigned char* sm, uint64_t* full,
                                              unsigned int* err, bool& ok) {
  const int slot = j % kRing;
  if (!mbar_wait(&full[slot], (uint32_t)((j / kRing) & 1), err)) ok = false;
  return smem_u32(sm + kNOffRing + slot * kW128);
}

// LayerNorm of a 128-wide row whose 32-column parts are held by the four
// threads (column groups) of one TMEM lane: partial sums through shared
// memory, combined in a fixed order.
__device__ __forceinline__ void row_layer_norm(float (&x)[32], const float* g, const float* bb,
                                               float (*red)[4][128], int cg, int row) {
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < 32; ++c) s += x[c];
  red[0][cg][row] = s;
  __syncthreads();
  const float mean = ((red[0][0][row] + red[0][1][row]) + (red[0][2][row] + red[0][3][row])) *
                     (1.0f / 128.0f);
  float v = 0.0f;
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    x[c] -= mean;
    v += x[c] * x[c];
  }
  red[1][cg][row] = v;
  __syncthreads();
  const float var = ((red[1][0][row] + red[1][1][row]) + (red[1][2][row] + red[1][3][row])) *
                    (1.0f / 128.0f);
  const float inv = 1.0f / sqrtf(var + kLnEps);
#pragma unroll
  for (int c = 0; c < 32; ++c) x[c] = x[c] * inv * g[cg * 32 + c] + bb[cg * 32 + c];
}

// 32 fp32 values of one row as fp16 into a SW128 [128 rows x 128] operand.
__device__ __forceinline__ void store_row16(unsigned char* op, const float (&x)[32], int row,
                                            int cg) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 h = __floats2half2_rn(x[8 * u + 2 * i], x[8 * u + 2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(op + sw128_offset(row, cg * 32 + 8 * u, 128)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void __launch_bounds__(kTfThreads, 1) tf_node_tc_kernel(const __grid_constant__ TfNodeArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float (*red)[4][128] = reinterpret_cast<float (*)[4][128]>(sm + kNOffRed);
  float* HeadS = reinterpret_cast<float*>(sm + kNOffHead);
  __shared__ uint64_t full[kRing];
  __shared__ uint64_t bar_mma;
  __shared__ uint32_t tmem_base;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, cg = warp >> 2;   // row quadrant, 32-column group
  const int row = quad * 32 + lane;
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
  const int64_t tiles = (p.rows + 127) / 128;
  const bool last = p.layer == 2;
  const int per_tile = last ? 13 : 15;
  const uint32_t idesc = idesc_h(128, 128);

  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) mbar_init(&full[i], 1);
    mbar_init(&bar_mma, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  if (last)
    for (int e = tid; e < kV * kH; e += kTfThreads) {
      const int v = e / kH, ff = e % kH;
      HeadS[e] = p.headT[ff * kV + v];
    }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;
  int64_t my_tiles = 0;
  if ((int64_t)blockIdx.x < tiles) my_tiles = (tiles - 1 - blockIdx.x) / gridDim.x + 1;
  Ring rg{0, 0, (int)(my_tiles * per_tile)};
  if (tid == 0) ring_issue(rg, sm, full, p, per_tile);
  bool ok = true;
  uint32_t ph = 0;
  int j = 0;   // next weight tile to consume (same on all threads)
  unsigned char* Aop = sm + kNOffA;

  auto mma_wait = [&]() {
    if (!mbar_wait(&bar_mma, ph, p.err)) ok = false;
    ph ^= 1;
    tc_fence_after();
  };

  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    if (__syncthreads_or(!ok)) break;
    const int64_t q = t * 128 + row;
    const bool valid = q < p.rows;
    int res = 0, K = 0;
    float m = 0.0f;
    if (valid) {
      res = p.row_res[q];
      const int L = p.bv.prot_len[p.bv.res_prot[res]];
      K = L < kK ? L : kK;
      m = p.mask[res];
    }
    float x[32];
    {
      const float* hrow = p.layer == 0 ? p.h_enc + (int64_t)res * kH : p.h + q * kH;
      const float4* h4 = reinterpret_cast<const float4*>(hrow + cg * 32);
      const float4* s4 = reinterpret_cast<const float4*>(p.S + q * kH + cg * 32);
      float sv[32];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 hv = valid ? h4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 svv = valid ? s4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        x[4 * i] = hv.x; x[4 * i + 1] = hv.y; x[4 * i + 2] = hv.z; x[4 * i + 3] = hv.w;
        sv[4 * i] = svv.x; sv[4 * i + 1] = svv.y; sv[4 * i + 2] = svv.z; sv[4 * i + 3] = svv.w;
      }
      store_row16(Aop, sv, row, cg);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- W3 after the slot sum, residual + LayerNorm 1 ----------------------
    if (tid == 0) {
      const uint32_t w = ring_wait(j, sm, full, p.err, ok);
      tc_fence_after();
      if (ok) mma_k128(tm + kNColD, smem_u32(Aop), w, 128, idesc, false);
      mma_commit(&bar_mma);
    }
    ++j;
    mma_wait();
    if (tid == 0) {
      rg.used = j;
      ring_issue(rg, sm, full, p, per_tile);
    }
    {
      float v[32];
      tmem_ld32(tm + lane_base + kNColD + (uint32_t)(cg * 32), v);
      const float Kf = (float)K;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        x[c] = x[c] + (v[c] + Kf * p.b3[cg * 32 + c]) * (1.0f / kMessageScale);
    }
    row_layer_norm(x, p.n1w, p.n1b, red, cg, row);   // x = h1
    tc_fence_before();
    store_row16(Aop, x, row, cg);   // W3's MMA has completed: the operand is free
    fence_async_smem();
    __syncthreads();
    // ---- FFN: DO = sum_i W_out[:, i] GELU(W_in[i] h1 + b_in[i]) ------------
    if (tid == 0) {
      uint32_t w = ring_wait(j, sm, full, p.err, ok);       // W_in[0]
      tc_fence_after();
      if (ok) mma_k128(tm + kNColIn, smem_u32(Aop), w, 128, idesc, false);
      w = ring_wait(j + 1, sm, full, p.err, ok);            // and its remainder
      tc_fence_after();
      if (ok) mma_k128(tm + kNColIn, smem_u32(Aop), w, 128, idesc, true);
      mma_commit(&bar_mma);
    }
    j += 2;
    mma_wait();
    for (int i = 0; i < 4; ++i) {
      unsigned char* F = sm + kNOffF + (i & 1) * kW128;
      {
        float v[32];
        tmem_ld32(tm + lane_base + kNColIn + (uint32_t)((i & 1) * 128 + cg * 32), v);
        float y[32];
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          const float2 g = gelu_tc_x2(make_float2(v[c] + p.bin[i * 128 + cg * 32 + c],
                                                  v[c + 1] + p.bin[i * 128 + cg * 32 + c + 1]));
          y[c] = g.x;
          y[c + 1] = g.y;
        }
        store_row16(F, y, row, cg);
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        rg.used = j;   // W_in[i] (and every earlier tile) is consumed
        ring_issue(rg, sm, full, p, per_tile);
        uint32_t w = ring_wait(j, sm, full, p.err, ok);   // W_out[:, i]
        tc_fence_after();
        if (ok) mma_k128(tm + kNColOut, smem_u32(F), w, 128, idesc, i > 0);
        if (i < 3) {
          const uint32_t din = tm + kNColIn + (uint32_t)(((i + 1) & 1) * 128);
          w = ring_wait(j + 1, sm, full, p.err, ok);      // W_in[i + 1]
          tc_fence_after();
          if (ok) mma_k128(din, smem_u32(Aop), w, 128, idesc, false);
          w = ring_wait(j + 2, sm, full, p.err, ok);      // and its remainder
          tc_fence_after();
          if (ok) mma_k128(din, smem_u32(Aop), w, 128, idesc, true);
        }
        mma_commit(&bar_mma);
      }
      j += i < 3 ? 3 : 1;
      mma_wait();
    }
    if (tid == 0) {
      rg.used = j;
      ring_issue(rg, sm, full, p, per_tile);
    }
    // ---- residual + LayerNorm 2, residue mask ------------------------------
    {
      float v[32];
      tmem_ld32(tm + lane_base + kNColOut + (uint32_t)(cg * 32), v);
#pragma unroll
      for (int c = 0; c < 32; ++c) x[c] = x[c] + v[c] + p.bout[cg * 32 + c];
    }
    row_layer_norm(x, p.n2w, p.n2b, red, cg, row);
#pragma unroll
    for (int c = 0; c < 32; ++c) x[c] = (m == 1.0f) ? x[c] : x[c] * m;
    tc_fence_before();
    if (!last) {
      // ---- the next layer's node terms: A = W1a h' + b1, PV = W1d h' -------
      if (valid) {
        float4* o = reinterpret_cast<float4*>(p.h + q * kH + cg * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          o[i] = make_float4(x[4 * i], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
      }
      store_row16(Aop, x, row, cg);
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        uint32_t w = ring_wait(j, sm, full, p.err, ok);
        tc_fence_after();
        if (ok) mma_k128(tm + kNColD, smem_u32(Aop), w, 128, idesc, false);
        w = ring_wait(j + 1, sm, full, p.err, ok);
        tc_fence_after();
        if (ok) mma_k128(tm + kNColIn, smem_u32(Aop), w, 128, idesc, false);
        mma_commit(&bar_mma);
      }
      j += 2;
      mma_wait();
      if (tid == 0) {
        rg.used = j;
        ring_issue(rg, sm, full, p, per_tile);
      }
      {
        float v[32];
        tmem_ld32(tm + lane_base + kNColD + (uint32_t)(cg * 32), v);
        if (valid) {
          float4* o = reinterpret_cast<float4*>(p.A_next + q * kH + cg * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            o[i] = make_float4(v[4 * i] + p.b1_next[cg * 32 + 4 * i],
                               v[4 * i + 1] + p.b1_next[cg * 32 + 4 * i + 1],
                               v[4 * i + 2] + p.b1_next[cg * 32 + 4 * i + 2],
                               v[4 * i + 3] + p.b1_next[cg * 32 + 4 * i + 3]);
        }
        tmem_ld32(tm + lane_base + kNColIn + (uint32_t)(cg * 32), v);
        if (valid) {
          uint4* o = reinterpret_cast<uint4*>(p.PV_next + q * kH + cg * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const __half2 h = __floats2half2_rn(v[8 * u + 2 * i], v[8 * u + 2 * i + 1]);
              w[i] = *reinterpret_cast<const uint32_t*>(&h);
            }
            o[u] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
    } else {
      // ---- logits (fp32) and the unscaled log-softmax -----------------------
      float (*part)[4][128] = reinterpret_cast<float (*)[4][128]>(sm + kNOffF);
#pragma unroll 1
      for (int v = 0; v < kV; ++v) {
        const float* hw = HeadS + v * kH + cg * 32;
        float z = 0.0f;
#pragma unroll
        for (int c = 0; c < 32; ++c) z = fmaf(x[c], hw[c], z);
        part[v][cg][row] = z;
      }
      __syncthreads();
      if (cg == 0 && valid) {
        float z[kV], mx = -INFINITY;
#pragma unroll
        for (int v = 0; v < kV; ++v) {
          z[v] = p.head_b[v] + ((part[v][0][row] + part[v][1][row]) +
                                (part[v][2][row] + part[v][3][row]));
          mx = fmaxf(mx, z[v]);
        }
        float sum = 0.0f;
#pragma unroll
        for (int v = 0; v < kV; ++v) sum += expf(z[v] - mx);
        const float ls = logf(sum);
        float* out = p.log_probs + q * kV;
#pragma unroll
        for (int v = 0; v < kV; ++v) out[v] = (z[v] - mx) - ls;
      }
    }
  }
  // Drain: no bulk copy may still be in flight when the CTA exits.
  if (tid == 0)
    for (int jj = j; jj < rg.issued; ++jj) {
      const int slot = jj % kRing;
      mbar_wait(&full[slot], (uint32_t)((jj / kRing) & 1), p.err);
    }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 512);
}

// pos[row of residue order[p]] = p and row -> residue, one CTA per sequence.
__global__ void tf_rows_kernel(BatchView bv, const int32_t* __restrict__ orders,
                               int* __restrict__ pos, int* __restrict__ row_res,
                               unsigned int* err) {
  const int sq = blockIdx.x;
  const int b = bv.seq_prot[sq];
  const int L = bv.prot_len[b];
  const int off = bv.prot_res_off[b];
  const int64_t q0 = bv.seq_row_off[sq];
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const int t = orders[q0 + i];
    if (t < 0 || t >= L) {
      atomicOr(err, kErrBadIndex);
    } else {
      pos[q0 + t] = i;
    }
    row_res[q0 + i] = off + i;
  }
}

}  // namespace

void launch_tf_rows(cudaStream_t st, const BatchView& bv, const int32_t* orders, int* pos,
                    int* row_res, unsigned int* err) {
  if (bv.num_sequences <= 0) return;
  tf_rows_kernel<<<bv.num_sequences, 256, 0, st>>>(bv, orders, pos, row_res, err);
}

void launch_tf_slot_tc(cudaStream_t st, const TfSlotArgs& p, int num_sms) {
  const int R = p.bv.total_residues;
  if (R <= 0) return;
  ensure_dynamic_smem((const void*)tf_slot_tc_kernel, (int)kSlotSmem);
  const int grid = R < num_sms ? R : num_sms;
  tf_slot_tc_kernel<<<grid, kTfThreads, kSlotSmem, st>>>(p);
}

void launch_tf_node_tc(cudaStream_t st, const TfNodeArgs& p, int num_sms) {
  const int64_t tiles = (p.rows + 127) / 128;
  if (tiles <= 0) return;
  ensure_dynamic_smem((const void*)tf_node_tc_kernel, (int)kNodeSmem);
  const int grid = (int)(tiles < num_sms ? tiles : num_sms);
  tf_node_tc_kernel<<<grid, kTfThreads, kNodeSmem, st>>>(p);
}

}  // namespace hkb
