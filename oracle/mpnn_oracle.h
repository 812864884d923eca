/* TEST INFRASTRUCTURE ONLY -- the CPU checker for the B200 design engine.
 *
 * A plain-C restatement of the ProteinMPNN v_48_020 design path of the
 * reference (megure-labs/hikoboshi, cpp/modules/mpnn/ + cpp/primitives/).
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * it; the product library never links or calls it.
 *
 * Weights are passed as 118 fp32 tensor pointers in this file's own slot order
 * (ORACLE_T_* below); the Python side binds them by safetensors name.  The
 * tensor set and shapes are the reference schema's
 * (cpp/include/hikoboshi/universal/detail/proteinmpnn_v48_020_schema.hpp:
 * 127-160).
 */
#ifndef HKB_MPNN_ORACLE_H
#define HKB_MPNN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORACLE_H = 128,
  ORACLE_KMAX = 48,
  ORACLE_V = 21,
  ORACLE_EDGE_IN = 416,
  ORACLE_FFN = 512,
  ORACLE_TENSORS = 118
};

/* Slot numbers. Encoder layer l tensors start at
 * ORACLE_T_ENC0 + 22*l in the order W1.w W1.b W2.w W2.b W3.w W3.b W11.w W11.b
 * W12.w W12.b W13.w W13.b norm1.w norm1.b norm2.w norm2.b norm3.w norm3.b
 * dense.W_in.w dense.W_in.b dense.W_out.w dense.W_out.b.  Decoder layer l
 * starts at ORACLE_T_DEC0 + 14*l: W1.w W1.b W2.w W2.b W3.w W3.b norm1.w
 * norm1.b norm2.w norm2.b dense.W_in.w dense.W_in.b dense.W_out.w
 * dense.W_out.b. */
enum {
  ORACLE_T_POS_W = 0,
  ORACLE_T_POS_B = 1,
  ORACLE_T_EDGE_W = 2,
  ORACLE_T_NORM_E_W = 3,
  ORACLE_T_NORM_E_B = 4,
  ORACLE_T_WE_W = 5,
  ORACLE_T_WE_B = 6,
  ORACLE_T_WS = 7,
  ORACLE_T_ENC0 = 8,
  ORACLE_T_DEC0 = 8 + 3 * 22,
  ORACLE_T_WOUT_W = 8 + 3 * 22 + 3 * 14,
  ORACLE_T_WOUT_B = 8 + 3 * 22 + 3 * 14 + 1
};

typedef struct {
  const float* t[ORACLE_TENSORS];
} oracle_weights;

/* CA kNN (knn_scalar semantics, include_self). idx/d2 are [L, K], K=min(48,L). */
int oracle_knn(const float* coords, const uint8_t* sources, int L,
               int32_t* idx, float* d2);

/* Edge features [L, K, 416] = [16 positional | 25 pairs x 16 RBF]. */
int oracle_edge_features(const oracle_weights* w, const float* coords,
                         const uint8_t* sources, int L, const int32_t* idx,
                         float* features);

/* Encoder: h_v [L,128], h_e [L,K,128], idx [L,K], mask [L]. h_e0 optional
 * [L,K,128] receives the edge embedding before the encoder layers. */
int oracle_encode(const oracle_weights* w, const float* coords,
                  const uint8_t* sources, int L, float* h_v, float* h_e,
                  int32_t* idx, float* mask, float* h_e0);

/* Random (use_input=0) or given (use_input=1, input_order may be NULL for
 * identity) decoding order. Returns 1 (InvalidArgument) on a non-permutation. */
int oracle_decode_order(const float* mask, int L, uint64_t seed, int use_input,
                        const int32_t* input_order, int32_t* order);

/* Teacher-forced scoring pass, unscaled log-softmax.  order: NULL -> random
 * from seed; else the given permutation. */
int oracle_teacher_forced(const oracle_weights* w, const float* coords,
                          const uint8_t* sources, int L, const int32_t* tokens,
                          const int32_t* order_in, uint64_t seed,
                          float* log_probs, int32_t* order_out, float* score);

/* Teacher-forced pass returning temperature-scaled log-probs
 * (logits / T, T := 1 when T <= 0 or non-finite), the quantity the
 * autoregressive sampler emits.  Used to check device decode output. */
int oracle_teacher_forced_scaled(const oracle_weights* w, const float* coords,
                                 const uint8_t* sources, int L,
                                 const int32_t* tokens, const int32_t* order,
                                 float temperature, float* log_probs);

/* One autoregressive design (proteinmpnn_inverse_fold_scalar semantics):
 * seed drives both the decoding order and the sampler stream. */
int oracle_inverse_fold(const oracle_weights* w, const float* coords,
                        const uint8_t* sources, int L, uint64_t seed,
                        float temperature, int n_to_c, const int32_t* order_in,
                        int32_t* tokens, float* log_probs, int32_t* order_out,
                        float* score);

/* The sampler's uniform stream: u_i for the i-th draw with the given seed. */
double oracle_uniform(uint64_t seed, int draw_index);

#ifdef __cplusplus
}
#endif
#endif
