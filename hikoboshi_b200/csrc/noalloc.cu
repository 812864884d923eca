// Allocation-free small-batch design: hkb_mpnn_design_noalloc.
//
// Who needs this: callers that must not allocate device memory while they
// run -- a plugin inside a host application whose GPU memory is owned by that
// application's pool allocator (a private cudaMalloc would fail or fragment
// the pool), or a latency-bound loop that cannot afford cudaMalloc's implicit
// device synchronisation.  They create the engine once (that allocates the
// weights), then design small batches here without any further allocation.
//
// All scratch lives in one file-scope __device__ array, g_noalloc_scratch, of
// fixed size (about 18 MiB).  Every GPU that loads the library holds its own
// copy until the process exits.  Host code must not hand the array's name to
// a kernel (on the host it is only a stand-in symbol): the first call on each
// device, with that device current, asks the runtime for the array's device
// address with cudaGetSymbolAddress and caches it.  That first call therefore
// does one-time set-up work and should come before any stream capture.
//
// Every call shares the array and leaves its contents behind.  Buffers that
// must start at zero are cleared at the start of each call.  Two calls whose
// GPU work overlaps (another host thread, another stream) race on the array.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "engine.hpp"
#include "host_order.hpp"

namespace hkb {
namespace {

constexpr int kMaxR = HKB_NOALLOC_MAX_RESIDUES;
constexpr int kMaxNS = HKB_NOALLOC_MAX_SEQUENCES;
constexpr int kMaxQ = HKB_NOALLOC_MAX_ROWS;
constexpr size_t kSL = (size_t)kMaxR * kK;

enum Buf {
  B_ERR, B_POFF, B_PLEN, B_RPROT, B_SPROT, B_SROW, B_G0, B_GC, B_SEED, B_TEMP,
  B_POS, B_EIDX, B_D2, B_MASK, B_HE, B_HV, B_FEAT, B_E1, B_EB, B_G1, B_NAC,
  B_SV, B_CNT, B_T3, B_H1, B_F, B_Y, B_PE0, B_PE1, B_PE2, B_PVE0, B_PVE1,
  B_PVE2, B_AENC0, B_PV, B_COUNT
};

constexpr size_t kBytes[B_COUNT] = {
    sizeof(unsigned int),               // B_ERR
    kMaxR * sizeof(int),                // B_POFF  (B <= R)
    kMaxR * sizeof(int),                // B_PLEN
    kMaxR * sizeof(int),                // B_RPROT
    kMaxNS * sizeof(int),               // B_SPROT
    kMaxNS * sizeof(int64_t),           // B_SROW
    kMaxNS * sizeof(int),               // B_G0
    kMaxNS * sizeof(int),               // B_GC
    kMaxNS * sizeof(uint64_t),          // B_SEED
    kMaxNS * sizeof(float),             // B_TEMP
    kMaxQ * sizeof(int),                // B_POS
    kSL * sizeof(int),                  // B_EIDX
    kSL * sizeof(float),                // B_D2
    kMaxR * sizeof(float),              // B_MASK
    kSL * kH * sizeof(float),           // B_HE
    (size_t)kMaxR * kH * sizeof(float), // B_HV
    kSL * kEdgeIn * sizeof(float),      // B_FEAT
    kSL * kH * sizeof(float),           // B_E1
    kSL * kH * sizeof(float),           // B_EB
    kSL * kH * sizeof(float),           // B_G1
    (size_t)kMaxR * 256 * sizeof(float),   // B_NAC
    (size_t)kMaxR * kH * sizeof(float),    // B_SV
    kMaxR * sizeof(float),                 // B_CNT
    (size_t)kMaxR * kH * sizeof(float),    // B_T3
    (size_t)kMaxR * kH * sizeof(float),    // B_H1
    (size_t)kMaxR * kFfn * sizeof(float),  // B_F
    (size_t)kMaxR * kH * sizeof(float),    // B_Y
    kSL * kH * sizeof(float),              // B_PE0
    kSL * kH * sizeof(float),              // B_PE1
    kSL * kH * sizeof(float),              // B_PE2
    (size_t)kMaxR * kH * sizeof(float),    // B_PVE0
    (size_t)kMaxR * kH * sizeof(float),    // B_PVE1
    (size_t)kMaxR * kH * sizeof(float),    // B_PVE2
    (size_t)kMaxR * kH * sizeof(float),    // B_AENC0
    2 * (size_t)kMaxQ * kH * sizeof(float) // B_PV
};

constexpr size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr size_t offset_of(int b) {
  size_t o = 0;
  for (int i = 0; i < b; ++i) o += align256(kBytes[i]);
  return o;
}

constexpr size_t kScratchBytes = offset_of(B_COUNT);
static_assert(kScratchBytes <= (size_t)20 << 20, "allocation-free scratch must stay modest");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_noalloc_scratch on `device` (which must be current).
hkb_status scratch_base(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (device < 0 || device >= 64) return {HKB_INVALID_ARGUMENT, "device ordinal out of range"};
  if (g_scratch_addr[device] == nullptr) {
    void* p = nullptr;
    const cudaError_t ce = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (ce != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return {HKB_INTERNAL_ERROR, "cudaGetSymbolAddress of the allocation-free scratch failed"};
    }
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
  return {HKB_OK, ""};
}

template <typename T>
T* at(unsigned char* base, Buf b) {
  return reinterpret_cast<T*>(base + offset_of(b));
}

#define NOALLOC_CUDA(call)                                                     \
  do {                                                                         \
    const cudaError_t ce_ = (call);                                            \
    if (ce_ != cudaSuccess) return {HKB_INTERNAL_ERROR, cudaGetErrorString(ce_)}; \
  } while (0)

}  // namespace
}  // namespace hkb

using namespace hkb;

extern "C" hkb_status hkb_mpnn_design_noalloc(hkb_engine* e, const hkb_design_batch* batch,
                                              hkb_design_out* out, void* stream) {
  if (e == nullptr || batch == nullptr || out == nullptr)
    return {HKB_INVALID_ARGUMENT, "engine, batch and output must be non-null"};
  if (out->tokens == nullptr || out->log_probs == nullptr || out->orders == nullptr ||
      out->scores == nullptr)
    return {HKB_INVALID_ARGUMENT, "allocation-free design needs device tokens, log_probs, orders and scores"};
  const int B = batch->num_proteins;
  if (B <= 0 || batch->residue_counts == nullptr || batch->num_seqs == nullptr)
    return {HKB_INVALID_ARGUMENT, "batch must contain at least one protein"};
  if (batch->coords == nullptr || batch->atom_sources == nullptr)
    return {HKB_INVALID_ARGUMENT, "inverse-fold structure must provide canonical backbone atoms"};
  int64_t R = 0, Q = 0, NS = 0;
  for (int b = 0; b < B; ++b) {
    const int L = batch->residue_counts[b];
    const int S = batch->num_seqs[b];
    if (L <= 0) return {HKB_INVALID_ARGUMENT, "inverse-fold structure must contain at least one residue"};
    if (S <= 0) return {HKB_INVALID_ARGUMENT, "inverse-fold num_seqs must be greater than zero"};
    const float T = batch->temperatures ? batch->temperatures[b] : 0.1f;
    if (!std::isfinite(T) || T < 0.0f)
      return {HKB_INVALID_ARGUMENT, "inverse-fold sampling_temp must be finite and >= 0"};
    R += L;
    NS += S;
    Q += (int64_t)S * L;
  }
  if (R > kMaxR || NS > kMaxNS || Q > kMaxQ)
    return {HKB_INVALID_ARGUMENT,
            "batch exceeds the allocation-free limits (at most 64 residues, 64 sequences and "
            "1024 designed residues per call)"};

  NOALLOC_CUDA(cudaSetDevice(e->device));
  unsigned char* base = nullptr;
  hkb_status s = scratch_base(e->device, &base);
  if (s.code != HKB_OK) return s;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e->stream;

  // Host tables, all on the stack.
  uint8_t hsrc[kMaxR * 5];
  int off[kMaxR], len[kMaxR], res_prot[kMaxR], seq_prot[kMaxNS], g0[kMaxNS], gc[kMaxNS];
  int64_t seq_row[kMaxNS];
  uint64_t seeds[kMaxNS];
  float temps[kMaxNS], mask[kMaxR];
  int32_t orders[kMaxQ];
  OrderKey keys[kMaxR];
  NOALLOC_CUDA(cudaMemcpyAsync(hsrc, batch->atom_sources, (size_t)R * 5, cudaMemcpyDeviceToHost, st));
  NOALLOC_CUDA(cudaStreamSynchronize(st));
  int r0 = 0, s0 = 0, max_len = 0, ng = 0;
  int64_t q0 = 0;
  for (int b = 0; b < B; ++b) {
    const int L = batch->residue_counts[b];
    const int S = batch->num_seqs[b];
    off[b] = r0;
    len[b] = L;
    max_len = std::max(max_len, L);
    for (int i = 0; i < L; ++i) {
      const uint8_t* a = hsrc + (size_t)(r0 + i) * 5;
      res_prot[r0 + i] = b;
      mask[r0 + i] = (a[0] && a[1] && a[2] && a[3]) ? 1.0f : 0.0f;
    }
    const int mode = batch->decode_orders ? batch->decode_orders[b] : HKB_DECODE_RANDOM;
    if (mode == HKB_DECODE_INPUT) {
      if (batch->input_orders == nullptr)
        return {HKB_INVALID_ARGUMENT, "ProteinMPNN input decoding_order must be a permutation"};
      bool seen[kMaxR] = {};
      for (int p = 0; p < L; ++p) {
        const int32_t r = batch->input_orders[r0 + p];
        if (r < 0 || r >= L || seen[r])
          return {HKB_INVALID_ARGUMENT, "ProteinMPNN input decoding_order must be a permutation"};
        seen[r] = true;
      }
    } else if (mode != HKB_DECODE_RANDOM && mode != HKB_DECODE_N_TO_C) {
      return {HKB_INVALID_ARGUMENT, "unknown decode order mode"};
    }
    for (int q = 0; q < S; ++q) {
      const int sq = s0 + q;
      seq_prot[sq] = b;
      seq_row[sq] = q0 + (int64_t)q * L;
      seeds[sq] = (batch->seeds ? batch->seeds[b] : 0ull) + (uint64_t)q;
      temps[sq] = batch->temperatures ? batch->temperatures[b] : 0.1f;
      int32_t* o = orders + seq_row[sq];
      if (mode == HKB_DECODE_RANDOM) random_decode_order_into(mask + r0, L, seeds[sq], keys, o);
      else if (mode == HKB_DECODE_N_TO_C) for (int p = 0; p < L; ++p) o[p] = p;
      else std::memcpy(o, batch->input_orders + r0, sizeof(int32_t) * L);
    }
    const int G = ar_f32_group_size();
    for (int q = 0; q < S; q += G) {
      g0[ng] = s0 + q;
      gc[ng] = std::min(G, S - q);
      ++ng;
    }
    r0 += L;
    s0 += S;
    q0 += (int64_t)S * L;
  }

  // Scratch carve-up and per-call initialisation.
  unsigned int* d_err = at<unsigned int>(base, B_ERR);
  int* d_poff = at<int>(base, B_POFF);
  int* d_plen = at<int>(base, B_PLEN);
  int* d_rprot = at<int>(base, B_RPROT);
  int* d_sprot = at<int>(base, B_SPROT);
  int64_t* d_srow = at<int64_t>(base, B_SROW);
  int* d_g0 = at<int>(base, B_G0);
  int* d_gc = at<int>(base, B_GC);
  uint64_t* d_seed = at<uint64_t>(base, B_SEED);
  float* d_temp = at<float>(base, B_TEMP);
  NOALLOC_CUDA(cudaMemcpyAsync(d_poff, off, sizeof(int) * B, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_plen, len, sizeof(int) * B, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_rprot, res_prot, sizeof(int) * R, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_sprot, seq_prot, sizeof(int) * NS, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_srow, seq_row, sizeof(int64_t) * NS, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_g0, g0, sizeof(int) * ng, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_gc, gc, sizeof(int) * ng, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_seed, seeds, sizeof(uint64_t) * NS, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(d_temp, temps, sizeof(float) * NS, cudaMemcpyHostToDevice, st));
  NOALLOC_CUDA(cudaMemcpyAsync(out->orders, orders, sizeof(int32_t) * Q, cudaMemcpyHostToDevice, st));
  float* h_v = at<float>(base, B_HV);
  float* PV = at<float>(base, B_PV);
  NOALLOC_CUDA(cudaMemsetAsync(d_err, 0, sizeof(unsigned int), st));
  NOALLOC_CUDA(cudaMemsetAsync(h_v, 0, sizeof(float) * R * kH, st));
  NOALLOC_CUDA(cudaMemsetAsync(PV, 0, kBytes[B_PV], st));

  BatchView bv;
  bv.num_proteins = B;
  bv.total_residues = (int)R;
  bv.total_rows = Q;
  bv.num_sequences = (int)NS;
  bv.prot_res_off = d_poff;
  bv.prot_len = d_plen;
  bv.res_prot = d_rprot;
  bv.seq_prot = d_sprot;
  bv.seq_row_off = d_srow;

  // Encoder (the same launches as the allocating path).
  const F32Weights& w = e->w32;
  const int64_t SL = R * kK;
  int* e_idx = at<int>(base, B_EIDX);
  float* d2 = at<float>(base, B_D2);
  float* dmask = at<float>(base, B_MASK);
  float* h_e = at<float>(base, B_HE);
  float* feat = at<float>(base, B_FEAT);
  float* E1 = at<float>(base, B_E1);
  float* EB = at<float>(base, B_EB);
  float* G1 = at<float>(base, B_G1);
  float* NAC = at<float>(base, B_NAC);
  float* Sv = at<float>(base, B_SV);
  float* cnt = at<float>(base, B_CNT);
  float* T3 = at<float>(base, B_T3);
  float* h1 = at<float>(base, B_H1);
  float* F = at<float>(base, B_F);
  float* Y = at<float>(base, B_Y);
  launch_knn(st, bv, batch->coords, batch->atom_sources, e_idx, d2, dmask, d_err, max_len);
  launch_edge_features(st, bv, w, batch->coords, batch->atom_sources, e_idx, feat);
  gemm_f32(st, SL, kH, kEdgeIn, feat, kEdgeIn, w.edge_wT, kH, nullptr, 0, E1, kH);
  launch_ln_rows(st, SL, E1, nullptr, nullptr, w.norm_e_w, w.norm_e_b, nullptr, nullptr, E1);
  gemm_f32(st, SL, kH, kH, E1, kH, w.We_T, kH, w.We_b, 0, h_e, kH);
  for (int l = 0; l < 3; ++l) {
    const auto& E = w.enc[l];
    gemm_f32(st, R, 256, kH, h_v, kH, E.W1acT, 256, E.b1ac, 0, NAC, 256);
    gemm_f32(st, SL, kH, kH, h_e, kH, E.W1bT, kH, nullptr, 0, EB, kH);
    launch_enc_msg_in(st, bv, NAC, EB, e_idx, G1);
    gemm_f32(st, SL, kH, kH, G1, kH, E.W2T, kH, E.b2, 1, EB, kH);
    launch_enc_aggregate(st, bv, EB, e_idx, dmask, Sv, cnt);
    gemm_f32(st, R, kH, kH, Sv, kH, E.W3T, kH, nullptr, 0, T3, kH);
    launch_enc_node_update(st, bv, T3, cnt, E.b3, h_v, E.n1w, E.n1b, h1);
    gemm_f32(st, R, kFfn, kH, h1, kH, E.WinT, kFfn, E.bin, 1, F, kFfn);
    gemm_f32(st, R, kH, kFfn, F, kFfn, E.WoutT, kH, nullptr, 0, Y, kH);
    launch_ln_rows(st, R, h1, Y, E.bout, E.n2w, E.n2b, dmask, nullptr, h_v);
    gemm_f32(st, R, 256, kH, h_v, kH, E.W11acT, 256, E.b11ac, 0, NAC, 256);
    gemm_f32(st, SL, kH, kH, h_e, kH, E.W11bT, kH, nullptr, 0, EB, kH);
    launch_enc_msg_in(st, bv, NAC, EB, e_idx, G1);
    gemm_f32(st, SL, kH, kH, G1, kH, E.W12T, kH, E.b12, 1, EB, kH);
    gemm_f32(st, SL, kH, kH, EB, kH, E.W13T, kH, E.b13, 0, G1, kH);
    launch_edge_ln_update(st, bv, G1, e_idx, E.n3w, E.n3b, h_e);
  }
  // Decoder tables.
  DecoderTables dt{};
  float* pe[3] = {at<float>(base, B_PE0), at<float>(base, B_PE1), at<float>(base, B_PE2)};
  float* pve[3] = {at<float>(base, B_PVE0), at<float>(base, B_PVE1), at<float>(base, B_PVE2)};
  for (int l = 0; l < 3; ++l) {
    gemm_f32(st, SL, kH, kH, h_e, kH, w.dec[l].W1bT, kH, nullptr, 0, pe[l], kH);
    gemm_f32(st, R, kH, kH, h_v, kH, w.dec[l].W1dT, kH, nullptr, 0, pve[l], kH);
    dt.PE[l] = pe[l];
    dt.PVenc[l] = pve[l];
  }
  float* a0 = at<float>(base, B_AENC0);
  gemm_f32(st, R, kH, kH, h_v, kH, w.dec[0].W1aT, kH, w.dec[0].b1, 0, a0, kH);
  dt.Aenc0 = a0;
  // Fused autoregressive decode and scores.
  ArArgs a{};
  a.group_seq0 = d_g0;
  a.group_count = d_gc;
  a.num_groups = ng;
  a.orders = out->orders;
  a.pos = at<int>(base, B_POS);
  a.tokens = out->tokens;
  a.log_probs = out->log_probs;
  a.scores = out->scores;
  a.PV = PV;
  a.seq_seed = d_seed;
  a.seq_temp = d_temp;
  a.mask = dmask;
  a.e_idx = e_idx;
  a.h_enc = h_v;
  a.total_rows = Q;
  launch_ar_decode_f32(st, bv, w, dt, a, d_err);
  launch_scores(st, bv, out->tokens, out->log_probs, dmask, out->scores);
  NOALLOC_CUDA(cudaGetLastError());

  unsigned int herr = 0;
  NOALLOC_CUDA(cudaMemcpyAsync(&herr, d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost, st));
  NOALLOC_CUDA(cudaStreamSynchronize(st));
  if (herr != 0) return {HKB_INTERNAL_ERROR, "device kernel saw an out-of-range index"};
  return {HKB_OK, ""};
}
