// Kernel launchers (host-callable) of the design engine.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace hkb {

// Raises `func`'s dynamic shared-memory limit to `bytes` on the current device,
// once per (device, kernel, size).  The attribute is per device, and engines on
// several devices or host threads launch the same kernels; the bookkeeping is
// guarded by a mutex.
void ensure_dynamic_smem(const void* func, int bytes);

// Per-call device tables describing a batch.
struct BatchView {
  int num_proteins = 0;
  int total_residues = 0;        // R
  int64_t total_rows = 0;        // Q = sum S_b L_b
  int num_sequences = 0;         // sum S_b
  const int* prot_res_off = nullptr;   // [B] first residue of protein b
  const int* prot_len = nullptr;       // [B]
  const int* res_prot = nullptr;       // [R] protein of residue
  const int* seq_prot = nullptr;       // [NS]
  const int64_t* seq_row_off = nullptr;  // [NS] first row of sequence in [Q]
};

// fp32 weights in the layouts the SIMT kernels read ("T" = [in][out]).
struct F32Weights {
  const float* pos_w;   // [16,66]
  const float* pos_b;   // [16]
  const float* edge_wT; // [416,128]
  const float* norm_e_w;
  const float* norm_e_b;
  const float* We_T;    // [128,128]
  const float* We_b;
  struct Enc {
    const float* W1acT;   // [128,256]  [W1a | W1c] for h_i and h_j terms
    const float* b1ac;    // [256]      [b1 | 0]
    const float* W1bT;    // [128,128]  h_E term
    const float* W2T; const float* b2;
    const float* W3T; const float* b3;
    const float* W11acT; const float* b11ac;
    const float* W11bT;
    const float* W12T; const float* b12;
    const float* W13T; const float* b13;
    const float* n1w; const float* n1b;
    const float* n2w; const float* n2b;
    const float* n3w; const float* n3b;
    const float* WinT;  const float* bin;   // [128,512]
    const float* WoutT; const float* bout;  // [512,128]
  } enc[3];
  struct Dec {
    const float* W1adT;   // [128,256]  [W1a | W1d]
    const float* b1ad;    // [256]      [b1 | 0]
    const float* W1aT;    // [128,128]  (view into W1adT rows is strided; kept separately)
    const float* b1;      // [128]
    const float* W1dT;    // [128,128]
    const float* W1bT;    // [128,128]
    const float* Stab;    // [21,128]  W1c . W_s[v]
    const float* W2T; const float* b2;
    const float* W3T; const float* b3;
    const float* n1w; const float* n1b;
    const float* n2w; const float* n2b;
    const float* WinT;  const float* bin;
    const float* WoutT; const float* bout;
  } dec[3];
  const float* headT;   // [128,21]
  const float* head_b;  // [21]
};

// Per-protein decoder tables produced by the decoder preparation.
struct DecoderTables {
  const float* PE[3];     // [R*48,128] W1b_l . h_E (no bias)
  const float* PVenc[3];  // [R,128]    W1d_l . h_enc
  const float* Aenc0;     // [R,128]    W1a_0 . h_enc + b1_0
};


// Generic fp32 GEMM: C[M,N] = act(A[M,K] . B[K,N] + bias[N]); act 0 none, 1 GELU.
void gemm_f32(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
              const float* B, int ldb, const float* bias, int act, float* C,
              int ldc);
// The packed-fp32 tiled form gemm_f32 uses when the shape allows (N a
// multiple of 128, K of 32, 16-byte aligned rows); out_f16 stores C as fp16.
bool gemm_f32x2_fits(int N, int K, const void* A, int lda, const void* B, int ldb,
                     const void* C, int ldc);
void gemm_f32x2(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
                const float* B, int ldb, const float* bias, int act, void* C, int ldc,
                bool out_f16);
// The same contraction on tcgen05 with both operands applied as fp16 value +
// fp16 remainder (three products): W given as value and remainder images
// (append_gemm_image layout, one 128-row block per 128 output columns), N a
// multiple of 128, K of 64, lda of 4; act 0 none, 1 GELU (fp32 output only).
void gemm_tc3(cudaStream_t st, int64_t M, int N, int K, const float* A, int lda,
              const unsigned char* Whi, const unsigned char* Wlo, const float* bias, int act,
              void* C, int ldc, bool out_f16, unsigned int* err);

// Largest protein one call accepts (kNN keeps one 8-byte key per candidate
// in shared memory and ranks every candidate against every other).
constexpr int kMaxResidues = 4096;

void launch_knn(cudaStream_t st, const BatchView& bv, const float* coords,
                const uint8_t* sources, int* e_idx, float* d2, float* mask,
                unsigned int* err, int max_len);

void launch_edge_features(cudaStream_t st, const BatchView& bv,
                          const F32Weights& w, const float* coords,
                          const uint8_t* sources, const int* e_idx, float* feat);

// out = LN(x + y (+ bias)) (* mask[row] if mask != null); rows of 128.
void launch_ln_rows(cudaStream_t st, int64_t rows, const float* x,
                    const float* y, const float* ybias, const float* g,
                    const float* b, const float* row_mask,
                    const int* row_to_mask, float* out);

// Encoder pieces.
void launch_enc_msg_in(cudaStream_t st, const BatchView& bv, const float* NAC,
                       const float* EB, const int* e_idx, float* G1);
void launch_enc_aggregate(cudaStream_t st, const BatchView& bv, const float* G2,
                          const int* e_idx, const float* mask, float* S,
                          float* cnt);
void launch_enc_node_update(cudaStream_t st, const BatchView& bv,
                            const float* T3, const float* cnt, const float* b3,
                            const float* h, const float* g, const float* b,
                            float* out);
void launch_edge_ln_update(cudaStream_t st, const BatchView& bv, const float* U3,
                           const int* e_idx, const float* g, const float* b,
                           float* h_e);
void launch_gather_rows(cudaStream_t st, int64_t rows, const int* row_res,
                        const float* src, float* dst);

// Teacher-forced pieces (rows = (sequence, residue) pairs of one chunk).
struct TfRows {
  int64_t rows = 0;
  const int* row_res = nullptr;       // [rows] global residue index
  const int64_t* row_seqbase = nullptr;  // [rows] row index of residue 0 of its sequence (chunk-local)
  const int* row_prot = nullptr;      // [rows]
  const int* pos = nullptr;           // [rows] position of the row's residue in its order
  const int* tokens = nullptr;        // [rows]
};
void launch_tf_slot_in(cudaStream_t st, const BatchView& bv, const TfRows& tr,
                       int layer, const float* AP, const DecoderTables& dt,
                       const float* Stab, const int* e_idx, float* G1);
void launch_row_slot_sum(cudaStream_t st, const BatchView& bv, const TfRows& tr,
                         const float* G2, float* S, float* kcount);
void launch_dec_node_update(cudaStream_t st, int64_t rows, const float* T3,
                            const float* kcount, const float* b3,
                            const float* h, const float* g, const float* b,
                            float* out);
void launch_log_softmax_rows(cudaStream_t st, int64_t rows, const float* logits,
                             float* out);

// Autoregressive decode (fused persistent kernel, fp32 SIMT).
struct ArArgs {
  const int* group_seq0;     // [groups] first global sequence of the group
  const int* group_count;    // [groups]
  int num_groups;
  const int* orders;         // [Q]
  int* pos;                  // [Q] scratch
  int* tokens;               // [Q] out
  float* log_probs;          // [Q,21] out
  float* scores;             // [NS] out
  float* PV;                 // [2,Q,128] scratch (zeroed by the caller)
  const uint64_t* seq_seed;  // [NS]
  const float* seq_temp;     // [NS]
  const float* mask;         // [R]
  const int* e_idx;          // [R,48]
  const float* h_enc;        // [R,128]
  int64_t total_rows;
};
void launch_ar_decode_f32(cudaStream_t st, const BatchView& bv,
                          const F32Weights& w, const DecoderTables& dt,
                          const ArArgs& a, unsigned int* err);

int ar_f32_group_size();

// ---- bf16 tensor-core path --------------------------------------------------
// Weight tiles for the fused decode kernel: every 128 x 128 operand tile is a
// 16-bit image already in the SW128 K-major shared-memory layout, and the
// tiles sit in the exact order the kernel consumes them in one decode position:
//   layer 0: W2, W3, (W_in[i], W_in[i] remainder) for i = 0..3, then
//            W_out[:, i] for i = 0..3                             (14 tiles)
//   then for l = 1, 2: W1a_l, W1d_l and the same 14               (16 each)
// W_in is applied as hi + remainder (two MMAs into one accumulator): its
// 16-bit rounding is the largest single error source of the decoder.
constexpr int kStreamTilesPerStep = 46;
// Stream tile index of layer l's W2 (its W1a and W1d sit just before it for
// l > 0); W3 follows W2, then the four W_in[i] (hi, remainder) pairs and the
// four W_out[:, i].
__host__ __device__ constexpr int stream_w2_tile(int l) { return l == 0 ? 0 : 14 + 16 * (l - 1) + 2; }
__host__ __device__ constexpr int stream_w1a_tile(int l) { return 14 + 16 * (l - 1); }
constexpr int kTileBytes = 128 * 128 * 2;

// Logit head of the decode kernel: fp32, transposed, one padded row per
// vocabulary entry (a logit is a float4 walk along both operands; the 528-byte
// pitch spreads eight consecutive entries over all 32 banks).
constexpr int kHeadPitch = 128 + 4;

struct Bf16DecodeWeights {
  const unsigned char* stream;  // [kStreamTilesPerStep][32 KiB]
  const float* headP = nullptr; // [21][kHeadPitch]
  const float* Stab[3];         // [21,128] W1c_l . W_s
  const float* b1[3];
  const float* b2[3];
  const float* b3[3];
  const float* n1w[3];
  const float* n1b[3];
  const float* n2w[3];
  const float* n2b[3];
  const float* bin[3];   // [512]
  const float* bout[3];
  const float* headT;    // [128,21] fp32
  const float* head_b;
};

struct Bf16DecodeTables {
  const uint16_t* PE[3];     // 16-bit [R*48,128] W1b_l h_E + PVenc_l[j] (DecTablesTcArgs)
  const uint16_t* PVenc[3];  // 16-bit [R,128] W1d_l h_enc
  const float* Aenc0;        // [R,128]
  const float* h_enc;        // [R,128]
};

struct ArBf16Args {
  const int* group_seqs;     // [num_groups, 16] sequence indices (same L per group)
  const int* group_count;
  int num_groups;
  const int* orders;
  int* pos;
  int* tokens;
  float* log_probs;          // [Q,21]: device memory or mapped pinned host memory
  float* lp_tok;             // [Q] log-prob of the sampled token (0 where masked)
  uint16_t* PV;              // 16-bit [2,Q,128] (rows written before they are read)
  const uint64_t* seq_seed;
  const float* seq_temp;
  const float* mask;
  const int* e_idx;
  int64_t total_rows;
  int stall_check = 0;       // failure-path check: wait on an unarmed barrier, then return
};

// Fused encoder-layer kernels (tensor-core modes; h_E fp16 [R*48,128]).
// NAC = [W1a h + b1 | W1c h] per residue, fp32 [R,256].
// Tensor map of a row-major [rows, 128] fp16 array (h_E) for 2-D TMA loads of
// [box_rows, 64] boxes with the 128-byte swizzle: one box lands as one
// 64-column atom of the SW128 K-major operand layout.  False if the driver
// cannot encode it.
bool make_rows_tensor_map(CUtensorMap* map, const uint16_t* base, int64_t rows, int box_rows);
constexpr int kNodeTileRows = 192;   // enc_node_tc: 4 residues x 48 slots per tile

struct EncNodeTcArgs {
  alignas(64) CUtensorMap map_he;       // h_E value, boxes of kNodeTileRows rows
  BatchView bv;
  const uint16_t* h_e = nullptr;
  const int* e_idx = nullptr;
  const float* mask = nullptr;
  const float* NAC = nullptr;
  const unsigned char* W1b = nullptr;   // fp16 SW128 images [128 out x 128 in]
  const unsigned char* W2 = nullptr;
  const unsigned char* W1b_lo = nullptr;   // their fp16 remainders (W - hi)
  const unsigned char* W2_lo = nullptr;
  const float* b2 = nullptr;
  float* S = nullptr;                   // [R,128] masked slot sums of GELU(W2 g + b2)
  float* cnt = nullptr;                 // [R] sum of m_i m_j
  unsigned int* err = nullptr;
};
void launch_enc_node_tc(cudaStream_t st, const EncNodeTcArgs& p, int num_sms);

struct EncEdgeTcArgs {
  alignas(64) CUtensorMap map_he;       // h_E value, boxes of 128 rows
  BatchView bv;
  const uint16_t* h_e = nullptr;        // read
  uint16_t* h_e_out = nullptr;          // written on slots with a valid neighbour (may alias)
  uint16_t* h_e_lo = nullptr;           // fp16 remainder of h_E (read and written in place)
  const int* e_idx = nullptr;
  const float* NAC = nullptr;           // [W11a h + b11 | W11c h]
  const unsigned char* W11b = nullptr;
  const unsigned char* W12 = nullptr;
  const unsigned char* W13 = nullptr;
  const unsigned char* W11b_lo = nullptr;   // fp16 remainders (W - hi)
  const unsigned char* W12_lo = nullptr;
  const unsigned char* W13_lo = nullptr;
  const float* b12 = nullptr;
  const float* b13 = nullptr;
  const float* n3w = nullptr;
  const float* n3b = nullptr;
  unsigned int* err = nullptr;
};
void launch_enc_edge_tc(cudaStream_t st, const EncEdgeTcArgs& p, int num_sms);

// Edge featurisation fused with the 416->128 edge linear, its LayerNorm and
// W_e: writes h_E (fp16 [R*48,128]) for every slot.
struct EncFeatTcArgs {
  BatchView bv;
  const float* coords = nullptr;        // [R,5,3]
  const uint8_t* src = nullptr;         // [R,5] atom sources (0 = missing)
  const int* e_idx = nullptr;
  const float* pos_w = nullptr;         // [16,66]
  const float* pos_b = nullptr;         // [16]
  const unsigned char* Wedge = nullptr; // fp16 SW128 image [128 x 448]
  const unsigned char* We = nullptr;    // fp16 SW128 image [128 x 128]
  const float* ln_w = nullptr;
  const float* ln_b = nullptr;
  const float* We_b = nullptr;
  uint16_t* h_e = nullptr;
  uint16_t* h_e_lo = nullptr;           // fp16 remainder of every h_E value
  unsigned int* err = nullptr;
};
void launch_enc_featurize_tc(cudaStream_t st, const EncFeatTcArgs& p, int num_sms);

// out[l] = h_E W[l]^T (fp16 [rows,128]) for three 128x128 images in one pass.
// Decoder slot tables of the fused decode kernel, one per layer l:
//   PE_l[s] = 16-bit(W1b_l h_E[s] + PVenc_l[j(s)])   (slot s = (residue, k))
// i.e. the edge term plus the encoder-state neighbour term of slot s, with the
// 16-bit PVenc_l row of the slot's neighbour j added in fp32 and the sum
// rounded once.  A slot whose neighbour is undecoded (and every slot at layer
// 0) reads only this row; a decoded neighbour adds the 16-bit correction
// W1d_l h_j - PVenc_l[j] that the decode kernel stores when it decodes j.
struct DecTablesTcArgs {
  alignas(64) CUtensorMap map_he;        // h_E value, boxes of 128 rows
  BatchView bv;
  const int* e_idx = nullptr;            // [R,48]
  const uint16_t* h_e = nullptr;
  int64_t rows = 0;
  const unsigned char* W[3] = {nullptr, nullptr, nullptr};
  const uint16_t* PVenc[3] = {nullptr, nullptr, nullptr};   // 16-bit [R,128]
  uint16_t* out[3] = {nullptr, nullptr, nullptr};
  unsigned int* err = nullptr;
};
void launch_dec_tables_tc(cudaStream_t st, const DecTablesTcArgs& p, int num_sms);

// Teacher-forced pass on tensor cores (fp16 engines); rows are the [Q]
// (sequence, residue) rows of the batch.
struct TfSlotArgs {
  BatchView bv;
  const int* prot_seq0 = nullptr;       // [B] first sequence of protein b
  const int* prot_nseq = nullptr;       // [B]
  int layer = 0;
  const uint16_t* h_e = nullptr;        // fp16 [R*48,128]
  const int* e_idx = nullptr;           // [R,48]
  const int* pos = nullptr;             // [Q] position of the row's residue in its order
  const int* tokens = nullptr;          // [Q]
  const float* Aenc0 = nullptr;         // [R,128] W1a_0 h_enc + b1_0 (layer 0)
  const uint16_t* PVenc = nullptr;      // fp16 [R,128] W1d_l h_enc
  const float* A = nullptr;             // [Q,128] W1a_l h + b1_l (layers 1, 2)
  const uint16_t* PV = nullptr;         // fp16 [Q,128] W1d_l h (layers 1, 2)
  const float* Stab = nullptr;          // [21,128] W1c_l W_s
  const unsigned char* W1b = nullptr;   // fp16 SW128 images [128 out x 128 in]
  const unsigned char* W2 = nullptr;
  const float* b2 = nullptr;
  float* S = nullptr;                   // [Q,128] out: sum_k GELU(W2 g + b2)
  unsigned int* err = nullptr;
};
void launch_tf_slot_tc(cudaStream_t st, const TfSlotArgs& p, int num_sms);

struct TfNodeArgs {
  BatchView bv;
  int64_t rows = 0;                     // Q
  int layer = 0;
  const int* row_res = nullptr;         // [Q] global residue of the row
  const float* mask = nullptr;          // [R]
  const float* h_enc = nullptr;         // [R,128] layer-0 residual
  float* h = nullptr;                   // [Q,128] residual in (layers 1, 2), h' out
  const float* S = nullptr;             // [Q,128]
  const unsigned char* stream = nullptr;  // decode weight tiles (kStreamTilesPerStep)
  int tile_ids[15] = {};                // W3, (W_in i, W_in i rem., W_out i) x 4, W1a', W1d'
  const float* b3 = nullptr;
  const float* n1w = nullptr;
  const float* n1b = nullptr;
  const float* bin = nullptr;           // [512]
  const float* bout = nullptr;
  const float* n2w = nullptr;
  const float* n2b = nullptr;
  const float* b1_next = nullptr;
  float* A_next = nullptr;              // [Q,128]
  uint16_t* PV_next = nullptr;          // fp16 [Q,128]
  const float* headT = nullptr;         // [128,21] (last layer)
  const float* head_b = nullptr;
  float* log_probs = nullptr;           // [Q,21] unscaled (last layer)
  unsigned int* err = nullptr;
};
void launch_tf_node_tc(cudaStream_t st, const TfNodeArgs& p, int num_sms);
void launch_tf_rows(cudaStream_t st, const BatchView& bv, const int32_t* orders, int* pos,
                    int* row_res, unsigned int* err);

int ar_tc_group_size();
// f32 -> fp16 (f16 = true) or bf16, round to nearest even.
void convert_f32_to_16(cudaStream_t st, const float* src, uint16_t* dst, int64_t n, bool f16);
// bf16 engines: dst[s] = 16-bit(PE[s] + PVenc[j(s)]) from the fp32 edge table
// (the slot tables of DecTablesTcArgs, built from fp32 products).
void presum_slot_table(cudaStream_t st, const BatchView& bv, const int* e_idx, const float* PE,
                       const uint16_t* PVenc, uint16_t* dst, bool f16);
void launch_ar_decode_tc(cudaStream_t st, const BatchView& bv,
                         const Bf16DecodeWeights& w, const Bf16DecodeTables& t,
                         const ArBf16Args& a, bool f16, unsigned int* err);

// Per-sequence decoding orders on the device (decode_order_scalar.cpp:61-116);
// modes[b]: 0 random, 1 identity, 2 input_orders[off_b ..].  Sequences whose
// random order the host must recompute (a score near a float rounding
// midpoint, or recheck_all) are appended to recheck_list.
struct OrderArgs {
  BatchView bv;
  const uint8_t* sources = nullptr;     // [R,5] atom sources (mask = N, CA, C, O present)
  const int* modes = nullptr;           // [B]
  const int32_t* input_orders = nullptr;  // [R] (mode 2 only)
  const uint64_t* seeds = nullptr;      // [NS]
  int32_t* orders = nullptr;            // [Q] out
  unsigned int* recheck_count = nullptr;
  int* recheck_list = nullptr;
  int recheck_cap = 0;
  int recheck_all = 0;
  unsigned int* err = nullptr;
};
void launch_decode_orders(cudaStream_t st, const OrderArgs& a);

// Mean NLL per sequence over unmasked residues.  With lp_tok ([Q], the
// sampled token's log-prob per row) the [Q,21] log_probs are not read.
void launch_scores(cudaStream_t st, const BatchView& bv, const int* tokens,
                   const float* log_probs, const float* mask, float* scores,
                   const float* lp_tok = nullptr);

}  // namespace hkb
