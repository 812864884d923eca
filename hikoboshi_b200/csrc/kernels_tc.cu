// Tensor-core throughput path: the fused persistent autoregressive decode
// kernel on tcgen05 tensor cores, with 16-bit operands (fp16 or bf16) and fp32
// accumulation, LayerNorm and softmax.
//
// One CTA owns up to 16 sequences of one protein and walks all L decode
// positions (inverse_fold_scalar.cpp:801-879).  Per position and DecLayer the
// dense work is restated so that every contraction is a 128-row tcgen05 MMA
// with the weights as the A operand (M = output features on TMEM lanes) and
// the activations as the B operand (N = sequences or neighbour slots on TMEM
// columns):
//   node terms   D_A = W1a h,  D_PV = W1d h          M=128 N=16  K=128
//   messages     D2  = W2 GELU(A_t + W1b h_E + W1d h_j + ...)
//                                                     M=128 N=48  K=128 (per sequence)
// W1b h_E + W1d h_enc_j is one precomputed 16-bit slot-table row per layer;
// a decoded neighbour j adds the 16-bit correction W1d (h_j - h_enc_j) this
// kernel stores when it decodes j, so an undecoded neighbour costs one
// gathered row instead of two.
//   aggregation  D3  = W3 (sum_k GELU(D2 + b2))       M=128 N=16  K=128
//   FFN          DF  = W_in[i] h1,  DO += W_out[:, i] GELU(DF + b_in)  (i = 0..3)
// W_in is applied as its fp16 value plus its fp16 remainder W_in - fp16(W_in)
// (two products summed in fp32: about twice the 16-bit precision for the
// decoder's most error-sensitive weight).  The slot sum runs along a thread's
// own TMEM row, LayerNorm statistics are warp reductions over a transposed
// fp32 copy, the logits are a warp per sequence, and the sampler is the
// reference's (double CDF).
//
// Weight tiles stream through a 4-slot shared-memory ring by 1-D bulk copies
// (no tensor map) issued by thread 0 in consumption order; independent MMAs
// of the node and FFN phases are issued by two threads.  The per-layer
// W1c W_s table is staged in shared memory by a bulk copy.  The CTA has 16
// warps.  In the message (slot) phase they form four groups of 4 warps; each
// group gathers the neighbour rows of its next sequence (in registers, one
// chunk ahead), builds the GELU operand, issues the MMA and sums
// GELU(D2 + b2) over the slots of its own sequences, so that one group's MMA
// wait and slot sum overlap the other groups' gathers and builds.  All 16
// warps share the node, LayerNorm, FFN and sampling phases.  Every wait is
// bounded; a timeout sets the error word and the CTA stops.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "kernels.hpp"
#include "tcgen05.cuh"

namespace hkb {
namespace {

using namespace tc;

constexpr int kGB = 16;           // sequences per CTA
// Message-phase groups: four groups of 4 warps, each owning one-sequence
// chunks (48 slots), measured slightly faster than two groups of 8 warps with
// two-sequence chunks (the other supported setting).
#ifndef HKB_MSG_GROUPS
#define HKB_MSG_GROUPS 4
#endif
constexpr int kGroups = HKB_MSG_GROUPS;   // message-phase groups (2 or 4)
constexpr int kChunkSeqs = 4 / kGroups;   // sequences per message MMA
constexpr int kChunkN = kChunkSeqs * kK;  // neighbour slots per message MMA
constexpr int kSlots = 4;         // weight ring depth
constexpr int kThreadsB = 512;
constexpr int kWarpsB = kThreadsB / 32;
constexpr int kGroupThreads = kThreadsB / kGroups;   // threads of a message group
static_assert(kGroups * kChunkN * 256 == 2 * 96 * 256, "message operand buffers");

// TMEM columns (fp32 accumulators, lanes = output features)
// (group g's message accumulator at kColD2 + g * kD2Stride: 96-column
// chunks sit back to back, 48-column ones on 64-column boundaries)
constexpr uint32_t kD2Stride = kChunkN == 96 ? 96 : 64;
constexpr uint32_t kColD2 = 0;
constexpr uint32_t kColA = kColD2 + kGroups * kD2Stride;
constexpr uint32_t kColPV = kColA + 16;
constexpr uint32_t kColD3 = kColPV + 16;
constexpr uint32_t kColDO = kColD3 + 16;
constexpr uint32_t kColDF = kColDO + 16;   // 4 x 16: W_in[i] h1 (hi product), i = 0..3
constexpr uint32_t kColDF2 = kColDF + 64;  // 4 x 16: the W_in[i] remainder products
constexpr uint32_t kTmemCols = 512;
static_assert(kColDF2 + 64 <= kTmemCols, "tensor memory columns");

// Shared memory map (offsets from a 1024-byte aligned base)
constexpr uint32_t kOffW = 0;                                   // 4 x 32 KiB
constexpr uint32_t kOffG1 = kOffW + kSlots * kTileBytes;        // 2 x 96 x 256 B
constexpr uint32_t kG1Bytes = kChunkN * 256;
constexpr uint32_t kOffHb = kOffG1 + kGroups * kG1Bytes;        // [16,128] bf16
constexpr uint32_t kOffSb = kOffHb + 4096;
constexpr uint32_t kOffH1b = kOffSb + 4096;
// The four FFN operands GELU(W_in[i] h1 + b_in[i]) ([16,128] each) live in the
// first message operand buffer, which is idle from the last message MMA of a
// layer to the first build of the next.
constexpr uint32_t kOffFb = kOffG1;
constexpr uint32_t kOffH = kOffH1b + 4096;                      // fp32 [16,128]
constexpr uint32_t kOffAa = kOffH + kGB * kH * 4;
// The residual of LayerNorm 1 (fp32 [16,128]) lives in the second message
// operand buffer, idle from the last message MMA of a layer to the first
// build of the next (it is written after W3 and last read at LayerNorm 2).
constexpr uint32_t kOffXs = kOffG1 + 4 * 4096;
// W1c_l W_s (fp32 [21,128]) of the current layer, staged by one bulk copy
// after the previous layer's last build.
constexpr uint32_t kStabBytes = kV * kH * 4;
constexpr uint32_t kOffStab = kOffAa + kGB * kH * 4;
constexpr uint32_t kOffNb = kOffStab + kStabBytes;              // int [16,48]
// The logit head (fp32, transposed with a padded pitch) is read from global
// memory through L1.
constexpr uint32_t kOffNbNext = kOffNb + kGB * kK * 4;          // int [16,48] next position
constexpr uint32_t kOffMisc = kOffNbNext + kGB * kK * 4;
constexpr uint32_t kSmemBytes = kOffMisc + 1024 + 1024;         // + misc + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "decode kernel shared memory");

struct Misc {
  uint64_t full[kSlots];
  uint64_t bar_d2[kGroups];   // message MMA of group g's chunk complete (D2 buffer g full)
  uint64_t bar_all;
  uint64_t bar_two;       // two issuing threads' MMAs complete (node terms)
  uint64_t bar_in[4];     // W_in[i] hi and remainder products complete (2 arrivals)
  uint64_t bar_ffn;       // the four W_out products complete
  uint64_t bar_stab;      // the next layer's W1c W_s table has landed
  uint32_t tbase;
  int abort_flag;
  int t[kGB];
  float m[kGB];
  long long qrow[kGB];
  unsigned long long rng[kGB];
  float temp[kGB];
  int off[kGB];   // first residue row of the sequence's protein
  int t_next[kGB];     // next position's residue and mask (prefetched)
  float m_next[kGB];
  int tok_cur[kGB];    // token sampled at the current position
};
static_assert(sizeof(Misc) <= 1024, "misc block");

template <bool F16>
__device__ __forceinline__ uint32_t pack16(float a, float b) {
  if constexpr (F16) {
    const __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}

template <bool F16>
__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (F16) {
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    } else {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
}

template <bool F16>
__device__ __forceinline__ uint16_t to16(float a) {
  return (uint16_t)(pack16<F16>(a, 0.0f) & 0xFFFFu);
}

template <bool F16>
__device__ __forceinline__ float from16(uint16_t h) {
  if constexpr (F16) return __half2float(__ushort_as_half(h));
  else return __uint_as_float((uint32_t)h << 16);
}

// Instruction descriptor for fp16 (format 0) or bf16 (format 1) operands.
template <bool F16>
__host__ __device__ constexpr uint32_t idesc16(int M, int N) {
  return F16 ? (idesc_bf16(M, N) & ~((7u << 7) | (7u << 10))) : idesc_bf16(M, N);
}

__device__ __forceinline__ unsigned long long splitmix_next(unsigned long long& s) {
  unsigned long long z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Thread-0 state of the weight-tile stream.  32-bit counters (at most
// 4096 x 46 tiles): the slot and tile indices are taken modulo 4 and 46 on
// every issue, on thread 0's critical path, and 64-bit remainders cost
// several times more.
struct Stream {
  int issued;   // tiles whose loads were issued
  int used;     // tiles released (their MMAs complete)
  int total;    // tiles this CTA consumes
};

__device__ __forceinline__ void stream_issue(Stream& s, unsigned char* sm, Misc& M,
                                             const unsigned char* img) {
  // Issue loads while a slot is free: tile j may load once tile j - kSlots is
  // released (its MMAs complete, tracked by `used` after a commit wait).
  while (s.issued < s.total && s.issued < s.used + kSlots) {
    const int slot = s.issued % kSlots;
    const int tile = s.issued % kStreamTilesPerStep;
    mbar_arrive_expect_tx(&M.full[slot], kTileBytes);
    bulk_g2s(sm + kOffW + slot * kTileBytes, img + (size_t)tile * kTileBytes, kTileBytes,
             &M.full[slot]);
    ++s.issued;
  }
}

// Waits until tile `j` is resident; returns its shared address.
__device__ __forceinline__ uint32_t stream_wait(int j, unsigned char* sm, Misc& M,
                                                unsigned int* err) {
  const int slot = j % kSlots;
  if (!mbar_wait(&M.full[slot], (uint32_t)((j / kSlots) & 1), err))
    *reinterpret_cast<volatile int*>(&M.abort_flag) = 1;
  return smem_u32(sm + kOffW + slot * kTileBytes);
}

template <bool F16>
__global__ void __launch_bounds__(kThreadsB, 1) ar_decode_tc_kernel(
    const __grid_constant__ BatchView bv, const __grid_constant__ Bf16DecodeWeights w,
    const __grid_constant__ Bf16DecodeTables tb, const __grid_constant__ ArBf16Args a,
    unsigned int* err) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Misc& M = *reinterpret_cast<Misc*>(sm + kOffMisc);
  float (*hS)[kH] = reinterpret_cast<float (*)[kH]>(sm + kOffH);
  float (*Aa)[kH] = reinterpret_cast<float (*)[kH]>(sm + kOffAa);
  float (*Xs)[kH] = reinterpret_cast<float (*)[kH]>(sm + kOffXs);
  int (*Nb)[kK] = reinterpret_cast<int (*)[kK]>(sm + kOffNb);
  int (*NbNext)[kK] = reinterpret_cast<int (*)[kK]>(sm + kOffNbNext);
  const float* HeadS = w.headP;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3;             // TMEM lane quadrant
  const int wg = warp >> 2;              // warpgroup 0..3
  const int feat = quad * 32 + lane;     // output feature this thread reads
  const uint32_t lane_base = (uint32_t)(quad * 32) << 16;

  const int g = blockIdx.x;
  // A group holds up to 16 sequences of proteins that share one length L
  // (possibly several proteins); each sequence keeps its protein's residue
  // offset.
  const int* gseq = a.group_seqs + (int64_t)g * kGB;
  const int n = a.group_count[g];
  const int b = bv.seq_prot[gseq[0]];
  const int L = bv.prot_len[b];
  const int K = L < kK ? L : kK;

  // Failure-path check (a.stall_check): wait, with the normal bounded wait, on
  // a barrier that nothing ever arrives on.  The wait gives up after about a
  // second, records kErrTimeout and the CTA returns before it allocates tensor
  // memory or issues any copy, so the caller sees InternalError and the context
  // stays usable.
  if (a.stall_check) {
    if (tid == 0) {
      mbar_init(&M.bar_all, 1);
      fence_barrier_init();
      mbar_wait(&M.bar_all, 0, err);
    }
    __syncthreads();
    return;
  }

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&M.full[i], 1);
    for (int i = 0; i < kGroups; ++i) mbar_init(&M.bar_d2[i], 1);
    mbar_init(&M.bar_all, 1);
    mbar_init(&M.bar_two, 2);
    for (int i = 0; i < 4; ++i) mbar_init(&M.bar_in[i], 2);
    mbar_init(&M.bar_ffn, 1);
    mbar_init(&M.bar_stab, 1);
    M.abort_flag = 0;
    fence_barrier_init();
  }
  if (tid < kGB) {
    const bool live = tid < n;
    const int sq = live ? gseq[tid] : 0;
    M.qrow[tid] = live ? bv.seq_row_off[sq] : 0;
    M.rng[tid] = live ? a.seq_seed[sq] : 0ull;
    M.temp[tid] = live ? a.seq_temp[sq] : 1.0f;
    M.off[tid] = live ? bv.prot_res_off[bv.seq_prot[sq]] : 0;
  }
  // Zero the small operand tiles once (rows of absent sequences stay zero).
  for (int e = tid; e < 3 * 4096 / 16; e += kThreadsB)
    reinterpret_cast<uint4*>(sm + kOffHb)[e] = make_uint4(0, 0, 0, 0);
  if (warp == 0) {
    tmem_alloc(&M.tbase, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = M.tbase;   // TMEM base address

  Stream st{0, 0, L * kStreamTilesPerStep};
  if (tid == 0) stream_issue(st, sm, M, w.stream);
  // W1c_l W_s staging: one copy in flight at most, issued by thread 0 after
  // every build of the layer before it (layer 0 of position 0: here).
  auto stab_issue = [&](int layer) {
    mbar_arrive_expect_tx(&M.bar_stab, kStabBytes);
    bulk_g2s(sm + kOffStab, w.Stab[layer], kStabBytes, &M.bar_stab);
  };
  bool stab_pending = false;   // thread 0: a staging copy not yet waited for
  uint32_t ph_stab = 0;
  if (tid == 0) {
    stab_issue(0);
    stab_pending = true;
  }

  // decode positions of every residue of this CTA's sequences
  for (int s = 0; s < n; ++s)
    for (int p = tid; p < L; p += kThreadsB) {
      const int t = a.orders[M.qrow[s] + p];
      if (t < 0 || t >= L) {
        atomicOr(err, kErrBadIndex);
        continue;
      }
      a.pos[M.qrow[s] + t] = p;
    }
  __syncthreads();

  // a group thread owns one 8-feature column chunk of this many slot rows
  constexpr int kRowsPerThread = kChunkN * 16 / kGroupThreads;
  const int grp = tid / kGroupThreads;       // message-phase group
  const int gtid = tid % kGroupThreads;
  // sequence of a chunk this warp sums (two-sequence chunks: warps 4-7 of a
  // group take the second)
  const int sub = kChunkSeqs == 2 ? (warp >> 2) & 1 : 0;
  constexpr int kRowStride = kGroupThreads / 16;   // slot rows between a thread's rows
  // message-phase chunks (two sequences each): group g takes g, g+2, ...
  const int nch = (n + kChunkSeqs - 1) / kChunkSeqs;
  volatile int* abort_p = &M.abort_flag;
  uint4 raw_pe[kRowsPerThread], raw_v[kRowsPerThread];   // in-flight slot rows
  uint32_t d2_count = 0;   // this group's message MMAs waited for so far
  uint32_t ph_all = 0, ph_two = 0, ph_ffn = 0, ph_in = 0;
  int tile = 0;   // next tile to consume (same on all threads)

  // The next position's h_enc / Aenc0 rows (residue t_next of each sequence)
  // into a free [16,128] fp32 buffer by cp.async: 16 rows x 32 16-byte chunks,
  // one per thread; absent sequences are zero-filled.
  auto stage_next_rows = [&](float (*dst)[kH], const float* table) {
    const int s = tid >> 5, c = tid & 31;
    const bool live = s < n;
    const float* src = live ? table + (int64_t)(M.off[s] + M.t_next[s]) * kH + c * 4 : table;
    cp_async16(&dst[s][c * 4], src, live);
    cp_async_commit();
  };

  for (int p = 0; p < L; ++p) {
    // uniform exit: every thread takes the same branch
    if (__syncthreads_or(M.abort_flag)) break;
    // ---- per-position set-up ------------------------------------------------
    // Position 0 reads everything here; later positions take the residue, the
    // mask and the neighbour codes prefetched during the previous position's
    // last layer (only the token decoded there is filled in now).
    constexpr int kFresh = 1 << 30;   // neighbour decoded at the previous position
    if (p == 0) {
      if (tid < kGB) {
        int t = 0;
        float m = 0.0f;
        if (tid < n) {
          t = a.orders[M.qrow[tid] + p];
          t = (t < 0 || t >= L) ? 0 : t;
          m = a.mask[M.off[tid] + t];
        }
        M.t[tid] = t;
        M.m[tid] = m;
      }
      __syncthreads();
      for (int e = tid; e < n * kK; e += kThreadsB) {
        const int s = e / kK, k = e % kK;
        int code = 0;
        if (k < K) {
          const int64_t rt = M.off[s] + M.t[s];
          int j = a.e_idx[rt * kK + k];
          if (j < 0 || j >= L) {
            atomicOr(err, kErrBadIndex);
            j = M.t[s];
          }
          code = j;   // nothing is decoded before position 0
        }
        Nb[s][k] = code;
      }
    } else {
      if (tid < kGB) {
        M.t[tid] = M.t_next[tid];
        M.m[tid] = M.m_next[tid];
      }
      for (int e = tid; e < n * kK; e += kThreadsB) {
        const int s = e / kK, k = e % kK;
        int code = NbNext[s][k];
        if (code & kFresh) code = (code & ~kFresh) | (M.tok_cur[s] << 17);
        Nb[s][k] = code;
      }
      __syncthreads();
    }
    if (p == 0) {
      for (int e = tid; e < kGB * kH; e += kThreadsB) {
        const int s = e >> 7, f = e & 127;
        hS[s][f] = s < n ? tb.h_enc[(int64_t)(M.off[s] + M.t[s]) * kH + f] : 0.0f;
        Aa[s][f] = s < n ? tb.Aenc0[(int64_t)(M.off[s] + M.t[s]) * kH + f] : 0.0f;
      }
    } else {
      cp_async_wait_all();   // rows staged during the previous position's logits
    }
    // the next position's residue and mask, for the prefetch in layer 2
    if (tid < kGB) {
      int t = 0;
      float m = 0.0f;
      if (tid < n && p + 1 < L) {
        t = a.orders[M.qrow[tid] + p + 1];
        t = (t < 0 || t >= L) ? 0 : t;
        m = a.mask[M.off[tid] + t];
      }
      M.t_next[tid] = t;
      M.m_next[tid] = m;
    }
    __syncthreads();
    // The next position's raw neighbour indices (one 192-byte e_idx row per
    // sequence) into NbNext by cp.async; they land during layer 0's message
    // phase and next_codes() turns them into codes (the Nb fill above has
    // read NbNext already).
    if (p + 1 < L && tid < n * (kK / 4)) {
      const int s = tid / (kK / 4), c = tid % (kK / 4);
      cp_async16(&NbNext[s][c * 4], a.e_idx + (int64_t)(M.off[s] + M.t_next[s]) * kK + c * 4,
                 true);
    }
    cp_async_commit();

    // Row loads of one neighbour-slot chunk (a message group): a thread owns
    // one 8-feature column chunk (tid % 16) of six slot rows: the slot table
    // row (W1b h_E + W1d h_enc of the neighbour, 16-bit) and, for a decoded
    // neighbour at layers 1 and 2, its correction row W1d (h_j - h_enc_j).
    auto load_rows = [&](int c, int layer, uint4 (&pe_raw)[kRowsPerThread],
                         uint4 (&v_raw)[kRowsPerThread]) {
      const int c8 = tid & 15;
      const int r0 = gtid >> 4;
      const uint16_t* PE = tb.PE[layer];
      const uint16_t* PVl =
          layer > 0 ? a.PV + (int64_t)(layer - 1) * a.total_rows * kH : nullptr;
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
        const int r = r0 + kRowStride * i;
        const int s = c * kChunkSeqs + r / kK, k = r % kK;
        pe_raw[i] = make_uint4(0, 0, 0, 0);
        v_raw[i] = make_uint4(0, 0, 0, 0);
        if (s < n && k < K) {
          const int code = Nb[s][k];
          const int j = code & 0xFFFF;
          const bool bw = (code >> 16) & 1;
          const int64_t rt = M.off[s] + M.t[s];
          pe_raw[i] = ld_nc_noalloc_v4(PE + (rt * kK + k) * kH + c8 * 8);
          if (bw && layer > 0)   // written by this kernel: coherent load
            v_raw[i] = ld_noalloc_v4(PVl + (M.qrow[s] + j) * kH + c8 * 8);
        }
      }
    };
    // GELU(A_t + [W1b h_E + W1d h_enc_j] + dV + W1c W_s[tok]) into the SW128
    // operand of chunk c, where dV = W1d (h_j - h_enc_j) for a decoded
    // neighbour at layers 1 and 2 and 0 otherwise.  The table terms are
    // widened and added in fp32 (W1c W_s[tok] from the layer's fp32 table in
    // shared memory).
    auto build_operand = [&](int c, const float* StabL,
                             const uint4 (&pe_raw)[kRowsPerThread],
                             const uint4 (&v_raw)[kRowsPerThread]) {
      unsigned char* dst = sm + kOffG1 + grp * kG1Bytes;
      const int c8 = tid & 15;
      const int r0 = gtid >> 4;
      // one-sequence chunks: every row of this thread shares A_t's 8 features
      float4 ca0 = make_float4(0.f, 0.f, 0.f, 0.f), ca1 = ca0;
      if (kChunkSeqs == 1 && c < n) {
        ca0 = reinterpret_cast<const float4*>(Aa[c])[c8 * 2];
        ca1 = reinterpret_cast<const float4*>(Aa[c])[c8 * 2 + 1];
      }
#pragma unroll
      for (int i = 0; i < kRowsPerThread; ++i) {
        const int r = r0 + kRowStride * i;
        const int s = c * kChunkSeqs + r / kK, k = r % kK;
        uint4 outv = make_uint4(0, 0, 0, 0);
        if (s < n && k < K) {
          const int code = Nb[s][k];
          const bool bw = (code >> 16) & 1;
          const int tok = code >> 17;
          float pe[8];
          unpack8<F16>(pe_raw[i], pe);
          float2 t2[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) t2[q] = make_float2(pe[2 * q], pe[2 * q + 1]);
          if (bw) {
            // decoded neighbour: (table + correction) + W1c W_s[tok]; the
            // correction row is zero at layer 0 and for undecoded neighbours,
            // which skip both terms (the sums are the same)
            float pv[8];
            unpack8<F16>(v_raw[i], pv);
            const float4* st = reinterpret_cast<const float4*>(StabL + tok * kH) + c8 * 2;
            const float4 s0 = st[0], s1 = st[1];
            const float st8[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int q = 0; q < 4; ++q)
              t2[q] = __fadd2_rn(__fadd2_rn(t2[q], make_float2(pv[2 * q], pv[2 * q + 1])),
                                 make_float2(st8[2 * q], st8[2 * q + 1]));
          }
          const float4 a0 =
              kChunkSeqs == 1 ? ca0 : reinterpret_cast<const float4*>(Aa[s])[c8 * 2];
          const float4 a1 =
              kChunkSeqs == 1 ? ca1 : reinterpret_cast<const float4*>(Aa[s])[c8 * 2 + 1];
          const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          // the operand holds 2 GELU(x): the epilogue halves D2 when it adds
          // b2 (W2 is linear and a power-of-two scale is exact)
          float2 y[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            y[q] = gelu2_tc_x2(__fadd2_rn(make_float2(av[2 * q], av[2 * q + 1]), t2[q]));
          outv = make_uint4(pack16<F16>(y[0].x, y[0].y), pack16<F16>(y[1].x, y[1].y),
                            pack16<F16>(y[2].x, y[2].y), pack16<F16>(y[3].x, y[3].y));
        }
        *reinterpret_cast<uint4*>(dst + sw128_offset(r, c8 * 8, kChunkN)) = outv;
      }
    };
    load_rows(grp, 0, raw_pe, raw_v);          // this group's first chunk of layer 0

    for (int l = 0; l < 3; ++l) {
      if (__syncthreads_or(M.abort_flag)) break;
      // ---- node terms for l >= 1 (MMAs issued at the end of layer l-1) -----
      if (l > 0) {
        const float b1 = w.b1[l][feat];        // in flight during the wait
        if (!mbar_wait(&M.bar_two, ph_two, err)) *abort_p = 1;
        ph_two ^= 1;
        tc_fence_after();
        if (tid == 0) {
          st.used = tile;                       // W1a, W1d of this layer released
          stream_issue(st, sm, M, w.stream);
        }
        // warpgroups 0/1: A columns 0-7 / 8-15, needed by every build
        const int s0 = (wg & 1) * 8;
        if (wg < 2) {
          float v[8];
          tmem_ld8(tm + lane_base + kColA + s0, v);
#pragma unroll
          for (int q = 0; q < 8; ++q) Aa[s0 + q][feat] = v[q] + b1;
        }
        tc_fence_before();
        __syncthreads();
        // warpgroups 2/3 (the second message group, whose first chunk comes
        // second): PV columns, W1d h of the current residues.  Later
        // positions' backward slots read them as the correction to the slot
        // table's encoder term, W1d h_t - PVenc[t] (16-bit).  Nothing at this
        // position reads them and the next node MMA (end of this layer) is the
        // first to overwrite the columns, so the stores stay off the first
        // build's path.
        if (wg >= 2) {
          const uint16_t* PVe = tb.PVenc[l];
          float e[8], v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int s = s0 + q;
            e[q] = s < n ? from16<F16>(PVe[(int64_t)(M.off[s] + M.t[s]) * kH + feat]) : 0.0f;
          }
          tc_fence_after();
          tmem_ld8(tm + lane_base + kColPV + s0, v);
          // Every decoded row is stored (the operand row of a masked residue
          // is zero, so its node term is exactly 0, as the reference's zeroed
          // hidden state gives; its h_enc row is zero too): PV needs no
          // initialisation.
          uint16_t* PV = a.PV + (int64_t)(l - 1) * a.total_rows * kH;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int s = s0 + q;
            if (s < n) PV[(M.qrow[s] + M.t[s]) * kH + feat] = to16<F16>(v[q] - e[q]);
          }
        }
      }
      // ---- messages: gather + GELU -> W2 MMA -> GELU + slot sum ------------
      // kGroups groups; group g takes chunks g, g + kGroups, ... and owns
      // operand buffer g and D2 buffer g.  Per chunk a group builds the
      // operand from rows already in registers, one elected thread issues
      // the MMA, the group issues the row loads of its next chunk (chunk g
      // of the next layer after its last one; they stay in flight through
      // the W3 / FFN phases), then waits for D2 and sums GELU(D2 + b2) over
      // the slots.  While one group waits on its MMA or sums, the others
      // build, so the work overlaps without handing buffers across groups.
      {
        // The PE rows (W1b h_E: K contiguous rows per sequence) of the next
        // message phase -- layer l+1 here, or layer 0 at the next position --
        // are prefetched into L2 a whole layer ahead: the table is far larger
        // than L2 and each row is read once per sequence, so these gathers
        // would otherwise wait on DRAM.
        if (grp == 1 && gtid < n && (l < 2 || p + 1 < L)) {
          const int t = l < 2 ? M.t[gtid] : M.t_next[gtid];
          bulk_prefetch_l2(tb.PE[l < 2 ? l + 1 : 0] + (int64_t)(M.off[gtid] + t) * kK * kH,
                           (uint32_t)(K * kH * 2));
        }
        if (mbar_wait(&M.bar_stab, ph_stab, err)) stab_pending = false;
        else *abort_p = 1;
        ph_stab ^= 1;
        const float* StabL = reinterpret_cast<const float*>(sm + kOffStab);
        const float2 half2c = make_float2(0.5f, 0.5f);
        const float b2 = w.b2[l][feat];
        const float2 b2p = make_float2(b2, b2);
        const uint32_t d2col = kColD2 + grp * kD2Stride + sub * kK;
        uint32_t wa = 0;
        for (int c = grp; c < nch; c += kGroups) {
          // Operand / D2 buffer grp is free: this group waited for its last
          // MMA and read its D2 before arriving at the barrier below.
          build_operand(c, StabL, raw_pe, raw_v);
          fence_async_smem();
          named_bar_sync(1 + grp, kGroupThreads);
          if (gtid == 0) {
            if (c == grp) wa = stream_wait(tile, sm, M, err);
            tc_fence_after();
            if (!*abort_p)
              mma_k128(tm + kColD2 + grp * kD2Stride, wa,
                       smem_u32(sm + kOffG1 + grp * kG1Bytes), kChunkN,
                       idesc16<F16>(128, kChunkN), false);
            mma_commit(&M.bar_d2[grp]);
          }
          if (c + kGroups < nch) load_rows(c + kGroups, l, raw_pe, raw_v);
          else if (l < 2) load_rows(grp, l + 1, raw_pe, raw_v);
          if (!*abort_p && !mbar_wait_abortable(&M.bar_d2[grp], d2_count & 1, err, abort_p))
            *abort_p = 1;
          ++d2_count;
          tc_fence_after();
          // four interleaved partial sums (a 48-long dependent add chain
          // would dominate), combined in a fixed order: slot i adds into
          // partial i mod 4, i.e. lane i mod 2 of pair (i mod 4) / 2.
          // Slots past K add an exact zero.
          // (L >= 48, every full neighbourhood, takes the branch without the
          // per-slot tests).
          float2 acc[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};
          auto sum_pairs = [&](const float* v, int n_pairs, int i0, bool full) {
#pragma unroll
            for (int m = 0; m < n_pairs; ++m) {
              float2 gv = gelu2_tc_x2(__ffma2_rn(make_float2(v[2 * m], v[2 * m + 1]), half2c, b2p));
              if (!full) {
                if (i0 + 2 * m >= K) gv.x = 0.0f;
                if (i0 + 2 * m + 1 >= K) gv.y = 0.0f;
              }
              acc[m & 1] = __fadd2_rn(acc[m & 1], gv);
            }
          };
          {
            float v[32];
            tmem_ld32(tm + lane_base + d2col, v);
            if (K == kK) sum_pairs(v, 16, 0, true);
            else sum_pairs(v, 16, 0, false);
          }
          {
            float v[16];
            tmem_ld16(tm + lane_base + d2col + 32, v);
            if (K == kK) sum_pairs(v, 8, 32, true);
            else sum_pairs(v, 8, 32, false);
          }
          const float total = 0.5f * ((acc[0].x + acc[0].y) + (acc[1].x + acc[1].y));
          const int s = c * kChunkSeqs + sub;
          if (s < n)
            *reinterpret_cast<uint16_t*>(sm + kOffSb + sw128_offset(s, feat, kGB)) =
                to16<F16>(total);
          tc_fence_before();   // D2 reads ordered before the group's next MMA
        }
        fence_async_smem();                     // slot sums feed the W3 MMA
      }
      ++tile;                                   // W2 consumed
      if (l == 0) cp_async_wait_all();          // next position's e_idx rows
      __syncthreads();
      // every build of this layer is done: stage the next layer's table
      if (tid == 0 && (l < 2 || p + 1 < L) && !*abort_p) {
        stab_issue(l < 2 ? l + 1 : 0);
        stab_pending = true;
      }
      // ---- W3 after the slot sum, residual + LayerNorm 1 --------------------
      // This layer's epilogue biases, loaded while the W3 MMA runs (a load
      // issued after an MMA wait would put its latency on the critical path).
      const float b3 = w.b3[l][feat] * (float)K;
      const float b_in0 = w.bin[l][feat], b_in1 = w.bin[l][128 + feat];
      const float b_in2 = w.bin[l][256 + feat], b_in3 = w.bin[l][384 + feat];
      const float b_out = w.bout[l][feat];
      if (tid == 0) {
        const uint32_t wa = stream_wait(tile, sm, M, err);
        tc_fence_after();
        if (!*abort_p)
          mma_k128(tm + kColD3, wa, smem_u32(sm + kOffSb), kGB, idesc16<F16>(128, kGB), false);
        mma_commit(&M.bar_all);
        // W2's MMAs have completed; its slot's next tile is not needed before
        // the FFN, so the refill follows the W3 MMA instead of delaying it
        st.used = tile;
        stream_issue(st, sm, M, w.stream);
      }
      ++tile;                                   // W3
      if (!mbar_wait(&M.bar_all, ph_all, err)) *abort_p = 1;
      ph_all ^= 1;
      tc_fence_after();
      if (tid == 0) {
        st.used = tile;
        stream_issue(st, sm, M, w.stream);
      }
      {
        float v[4];
        tmem_ld4(tm + lane_base + kColD3 + wg * 4, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int s = wg * 4 + q;
          Xs[s][feat] = hS[s][feat] + (v[q] + b3) * (1.0f / kMessageScale);
        }
      }
      tc_fence_before();
      __syncthreads();
      for (int s = warp; s < kGB; s += kWarpsB) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = Xs[s][lane * 4 + u];
        warp_layer_norm128(x, w.n1w[l], w.n1b[l], lane);
#pragma unroll
        for (int u = 0; u < 4; ++u) Xs[s][lane * 4 + u] = x[u];   // h1 (fp32)
        uint2 pk = make_uint2(pack16<F16>(x[0], x[1]), pack16<F16>(x[2], x[3]));
        *reinterpret_cast<uint2*>(sm + kOffH1b + sw128_offset(s, lane * 4, kGB)) = pk;
      }
      fence_async_smem();
      __syncthreads();
      // ---- layer 0, while the first W_in products run: the next position's
      // neighbour codes (its residue and mask were read at this position's
      // set-up, its raw neighbour indices staged in NbNext then) and an L2
      // prefetch of its node rows; they are consumed after this position's
      // sampling.  The pos / tokens loads of a thread's entries are all
      // issued before any is used: one global-load round trip.
      auto next_codes = [&]() {
        constexpr int kPer = (kGB * kK + kThreadsB - 1) / kThreadsB;
        int jj[kPer], ps[kPer], tk[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int e = tid + kThreadsB * i;
          const int s = e / kK, k = e % kK;
          jj[i] = -1;
          ps[i] = 0;
          tk[i] = 0;
          if (e < n * kK && k < K) {
            int j = NbNext[s][k];
            if (j < 0 || j >= L) {
              atomicOr(err, kErrBadIndex);
              j = M.t_next[s];
            }
            jj[i] = j;
            const int64_t qj = M.qrow[s] + j;
            ps[i] = a.pos[qj];
            tk[i] = a.tokens[qj];   // used only if decoded before this position
          }
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int e = tid + kThreadsB * i;
          if (e < n * kK) {
            int code = 0;
            const int j = jj[i];
            if (j >= 0) {
              if (ps[i] < p) code = j | (1 << 16) | (tk[i] << 17);
              else if (ps[i] == p) code = j | (1 << 16) | kFresh;   // decoded at this position
              else code = j;
            }
            NbNext[e / kK][e % kK] = code;
          }
        }
        if (tid < n * 8) {
          const int s = tid >> 3, line = tid & 3;
          const float* row = ((tid >> 2) & 1 ? tb.Aenc0 : tb.h_enc) +
                             (int64_t)(M.off[s] + M.t_next[s]) * kH + line * 32;
          asm volatile("prefetch.global.L2 [%0];" ::"l"(row));
        }
      };
      // ---- FFN: DO = sum_i W_out[:, i] GELU(W_in[i] h1 + b_in[i]) ----------
      // The stream holds W_in[0..3] (hi, remainder) and then W_out[:, 0..3],
      // so the eight W_in products never wait for a GELU: thread 0 issues the
      // hi products, thread 32 the remainder products, chunk i into its own
      // TMEM columns, each pair completing bar_in[i].  Round 1 issues chunks
      // 0 and 1 (their tiles are resident by now), round 2 chunks 2 and 3
      // (their tiles load as chunks 0 and 1 complete), and every thread
      // applies GELU(i) as soon as bar_in[i] completes; after one barrier
      // thread 0 issues the four W_out products into DO.
      auto issue_in = [&](int i) {
        if (tid == 0 || tid == 32) {
          const int lo = tid == 32;
          const uint32_t wa = stream_wait(tile + 2 * i + lo, sm, M, err);
          tc_fence_after();
          if (!*abort_p)
            mma_k128(tm + (lo ? kColDF2 : kColDF) + 16 * i, wa, smem_u32(sm + kOffH1b), kGB,
                     idesc16<F16>(128, kGB), false);
          mma_commit(&M.bar_in[i]);
        }
      };
      auto gelu_in = [&](int i, float bi) {
        if (!mbar_wait(&M.bar_in[i], ph_in, err)) *abort_p = 1;
        tc_fence_after();
        if (tid == 0) {
          st.used = tile + 2 * (i + 1);         // W_in[0..i] and remainders consumed
          stream_issue(st, sm, M, w.stream);
        }
        float v[4], v2[4];
        tmem_ld4(tm + lane_base + kColDF + 16 * i + wg * 4, v);
        tmem_ld4(tm + lane_base + kColDF2 + 16 * i + wg * 4, v2);
        unsigned char* fb = sm + kOffFb + i * 4096;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int s = wg * 4 + q;
          const float y = s < n ? gelu_tc((v[q] + v2[q]) + bi) : 0.0f;
          *reinterpret_cast<uint16_t*>(fb + sw128_offset(s, feat, kGB)) = to16<F16>(y);
        }
      };
      issue_in(0);
      issue_in(1);
      if (l == 0 && p + 1 < L) next_codes();
      gelu_in(0, b_in0);
      gelu_in(1, b_in1);
      issue_in(2);
      issue_in(3);
      gelu_in(2, b_in2);
      gelu_in(3, b_in3);
      ph_in ^= 1;
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        for (int i = 0; i < 4; ++i) {
          const uint32_t wa = stream_wait(tile + 8 + i, sm, M, err);   // W_out[:, i]
          tc_fence_after();
          if (!*abort_p)
            mma_k128(tm + kColDO, wa, smem_u32(sm + kOffFb + i * 4096), kGB,
                     idesc16<F16>(128, kGB), i > 0);
        }
        mma_commit(&M.bar_ffn);
      }
      tile += 12;
      if (!mbar_wait(&M.bar_ffn, ph_ffn, err)) *abort_p = 1;
      ph_ffn ^= 1;
      tc_fence_after();
      if (tid == 0) {
        st.used = tile;
        stream_issue(st, sm, M, w.stream);
      }
      // ---- residual + LayerNorm 2, residue mask ------------------------------
      {
        float v[4];
        tmem_ld4(tm + lane_base + kColDO + wg * 4, v);
        const float bo = b_out;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int s = wg * 4 + q;
          Aa[s][feat] = Xs[s][feat] + v[q] + bo;   // Aa reused as LN2 input
        }
      }
      tc_fence_before();
      __syncthreads();
      for (int s = warp; s < kGB; s += kWarpsB) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = Aa[s][lane * 4 + u];
        warp_layer_norm128(x, w.n2w[l], w.n2b[l], lane);
        const float m = M.m[s];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          x[u] = (m == 1.0f) ? x[u] : x[u] * m;
          hS[s][lane * 4 + u] = x[u];
        }
        uint2 pk = make_uint2(pack16<F16>(x[0], x[1]), pack16<F16>(x[2], x[3]));
        *reinterpret_cast<uint2*>(sm + kOffHb + sw128_offset(s, lane * 4, kGB)) = pk;
      }
      fence_async_smem();
      __syncthreads();
      // ---- next layer's node terms: W1a h, W1d h ------------------------------
      if (l < 2) {
        if (tid == 0 || tid == 32) {   // W1a by thread 0, W1d by thread 32
          const uint32_t wa = stream_wait(tid == 0 ? tile : tile + 1, sm, M, err);
          tc_fence_after();
          if (!*abort_p)
            mma_k128(tm + (tid == 0 ? kColA : kColPV), wa, smem_u32(sm + kOffHb), kGB,
                     idesc16<F16>(128, kGB), false);
          mma_commit(&M.bar_two);
        }
        tile += 2;                              // W1a, W1d of layer l+1 (released
                                                // after the wait at its start)
      }
    }
    if (__syncthreads_or(M.abort_flag)) break;
    // Aa is free from here to the next position's set-up
    if (p + 1 < L) stage_next_rows(Aa, tb.Aenc0);
    // ---- logits and sampling ------------------------------------------------
    // One warp per sequence (kGB == kWarpsB).  Lane i holds features
    // 4i..4i+3 of h and forms its partial dot products with the 21 head rows
    // (coalesced 512-byte row reads); a reduce-scatter over the warp (five
    // butterfly levels, each lane keeping half of its values) leaves lane v
    // with the full product for vocabulary entry v.  Then
    // (sampler_scalar.cpp:49-92): temperature-scaled log-softmax emitted as
    // the log-prob row, then greedy argmax (first maximum) or one uniform draw
    // against the double-precision CDF.  Sums run as warp reductions, so they
    // differ from the serial order by rounding only.
    static_assert(kGB == kWarpsB, "one warp per sequence");
    if (warp < n) {
      const int s = warp;
      float zp[32];
      {
        const float4 h = reinterpret_cast<const float4*>(hS[s])[lane];
#pragma unroll
        for (int v = 0; v < 32; ++v) {
          zp[v] = 0.0f;
          if (v < kV) {
            const float4 wv = reinterpret_cast<const float4*>(HeadS + v * kHeadPitch)[lane];
            zp[v] = fmaf(h.w, wv.w, fmaf(h.z, wv.z, fmaf(h.y, wv.y, h.x * wv.x)));
          }
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
          const float send = up ? zp[i] : zp[i + o];
          const float keep = up ? zp[i + o] : zp[i];
          zp[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      const int t = M.t[s];
      const int64_t q = M.qrow[s] + t;
      float* lp = a.log_probs + q * kV;
      const bool in_vocab = lane < kV;
      int tok = kV - 1;
      float lpv = 0.0f;   // this lane's log-prob (0 for a masked residue)
      if (M.m[s] == 0.0f) {
        if (in_vocab) lp[lane] = 0.0f;
      } else {
        const float temperature = M.temp[s];
        const bool greedy = !(temperature > 0.0f);
        const float T = (temperature > 0.0f && isfinite(temperature)) ? temperature : 1.0f;
        const float z = in_vocab ? (w.head_b[lane] + zp[0]) / T : -INFINITY;
        const float mx = warp_max(z);
        const float e = in_vocab ? expf(z - mx) : 0.0f;
        const float sum = warp_sum(e);
        const float ls = logf(sum), inv = 1.0f / sum;
        lpv = in_vocab ? (z - mx) - ls : 0.0f;
        if (in_vocab) lp[lane] = lpv;
        if (greedy) {
          const unsigned top = __ballot_sync(0xffffffffu, in_vocab && z == mx);
          tok = top ? __ffs(top) - 1 : 0;
        } else {
          double u = 0.0;
          if (lane == 0) {
            unsigned long long r = M.rng[s];
            u = (double)(splitmix_next(r) >> 11) * (1.0 / 9007199254740992.0);
            M.rng[s] = r;
          }
          u = __shfl_sync(0xffffffffu, u, 0);
          double cum = in_vocab ? (double)(e * inv) : 0.0;
#pragma unroll
          for (int d = 1; d < 32; d <<= 1) {
            const double o = __shfl_up_sync(0xffffffffu, cum, d);
            if (lane >= d) cum += o;
          }
          const unsigned hit = __ballot_sync(0xffffffffu, in_vocab && u < cum);
          if (hit) tok = __ffs(hit) - 1;
        }
      }
      const float lpt = __shfl_sync(0xffffffffu, lpv, tok);
      if (lane == 0) {
        a.tokens[q] = tok;
        a.lp_tok[q] = lpt;
        M.tok_cur[s] = tok;
      }
    }
    // Warp w stages row w, the row it alone read above.
    __syncwarp();
    if (p + 1 < L) stage_next_rows(hS, tb.h_enc);
    __syncthreads();
  }
  cp_async_wait_all();   // staged rows of a position an abort skipped
  // Drain: no bulk copy may still be in flight when the CTA exits.
  if (tid == 0) {
    if (stab_pending) mbar_wait(&M.bar_stab, ph_stab, err);
    for (int j = tile; j < st.issued; ++j) {
      const int slot = j % kSlots;
      mbar_wait(&M.full[slot], (uint32_t)((j / kSlots) & 1), err);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, kTmemCols);
}

template <bool F16>
__global__ void f32_to_16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst,
                                 int64_t n) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
  if (i + 1 < n) {
    *reinterpret_cast<uint32_t*>(dst + i) = pack16<F16>(src[i], src[i + 1]);
  } else if (i < n) {
    dst[i] = to16<F16>(src[i]);
  }
}

}  // namespace

int ar_tc_group_size() { return kGB; }

// One thread per (slot, 8-feature chunk): dst = 16-bit(PE + PVenc[neighbour]).
template <bool F16>
__global__ void presum_slot_table_kernel(const BatchView bv, const int* __restrict__ e_idx,
                                         const float* __restrict__ PE,
                                         const uint16_t* __restrict__ PVenc,
                                         uint16_t* __restrict__ dst, int64_t units) {
  const int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const int64_t s = u >> 4;
  const int c = (int)(u & 15) * 8;
  const int r = (int)(s / kK), k = (int)(s % kK);
  const int b = bv.res_prot[r];
  const int L = bv.prot_len[b];
  const int j = k < (L < kK ? L : kK) ? e_idx[s] : -1;
  const int rj = (j >= 0 && j < L) ? bv.prot_res_off[b] + j : -1;
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[i] = PE[s * kH + c + i];
    if (rj >= 0) x[i] += from16<F16>(PVenc[(int64_t)rj * kH + c + i]);
  }
  *reinterpret_cast<uint4*>(dst + s * kH + c) =
      make_uint4(pack16<F16>(x[0], x[1]), pack16<F16>(x[2], x[3]), pack16<F16>(x[4], x[5]),
                 pack16<F16>(x[6], x[7]));
}

void presum_slot_table(cudaStream_t st, const BatchView& bv, const int* e_idx, const float* PE,
                       const uint16_t* PVenc, uint16_t* dst, bool f16) {
  const int64_t units = (int64_t)bv.total_residues * kK * 16;
  if (units <= 0) return;
  const unsigned grid = (unsigned)((units + 255) / 256);
  if (f16) presum_slot_table_kernel<true><<<grid, 256, 0, st>>>(bv, e_idx, PE, PVenc, dst, units);
  else presum_slot_table_kernel<false><<<grid, 256, 0, st>>>(bv, e_idx, PE, PVenc, dst, units);
}

void convert_f32_to_16(cudaStream_t st, const float* src, uint16_t* dst, int64_t n, bool f16) {
  if (n <= 0) return;
  const int64_t threads = (n + 1) / 2;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  if (f16) f32_to_16_kernel<true><<<grid, 256, 0, st>>>(src, dst, n);
  else f32_to_16_kernel<false><<<grid, 256, 0, st>>>(src, dst, n);
}

void launch_ar_decode_tc(cudaStream_t st, const BatchView& bv, const Bf16DecodeWeights& w,
                         const Bf16DecodeTables& t, const ArBf16Args& a, bool f16,
                         unsigned int* err) {
  if (a.num_groups <= 0) return;
  ensure_dynamic_smem((const void*)ar_decode_tc_kernel<true>, (int)kSmemBytes);
  ensure_dynamic_smem((const void*)ar_decode_tc_kernel<false>, (int)kSmemBytes);
  if (f16)
    ar_decode_tc_kernel<true><<<a.num_groups, kThreadsB, kSmemBytes, st>>>(bv, w, t, a, err);
  else
    ar_decode_tc_kernel<false><<<a.num_groups, kThreadsB, kSmemBytes, st>>>(bv, w, t, a, err);
}

}  // namespace hkb
