/* TEST INFRASTRUCTURE ONLY -- CPU checker for the B200 design engine.
 *
 * Plain-C restatement of the reference's ProteinMPNN v_48_020 design path
 * (megure-labs/hikoboshi).  Every function cites the reference file:line it
 * follows (paths relative to the reference repo).  Dense contractions
 * accumulate in double and round once, so this checker sits at least as close
 * to exact arithmetic as the reference's fp32 GEMMs; element-wise functions use
 * the reference's own published approximations (table + Taylor exp,
 * Abramowitz-Stegun 7.1.26 erf, Welford LayerNorm) so features and activations
 * agree to a few ulps.
 *
 * Never linked into, or called by, the product library.
 */
#include "mpnn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define H ORACLE_H
#define V ORACLE_V
#define FFN ORACLE_FFN
#define EDGE_IN ORACLE_EDGE_IN

/* ------------------------------------------------------------------------ */
/* Element-wise pieces                                                       */
/* ------------------------------------------------------------------------ */

/* exp(x) for x <= 0 by integer range reduction against a table of e^-n and a
 * 6th-order Taylor polynomial of the remainder; returns 0 below -16 and 1 for
 * positive input (cpp/include/hikoboshi/primitives/detail/fast_exp_neg.hpp:
 * 9-52). */
static float exp_neg_table[17];
static int exp_neg_ready = 0;

static void exp_neg_init(void) {
  if (exp_neg_ready) return;
  for (int n = 0; n <= 16; ++n) exp_neg_table[n] = (float)exp(-(double)n);
  exp_neg_ready = 1;
}

static float exp_neg(float x) {
  if (x != x) return x;
  float nx = -x;
  if (nx > 16.0f) return 0.0f;
  if (nx < 0.0f) nx = 0.0f;
  int n = (int)(nx + 0.5f);
  if (n > 16) n = 16;
  const float r = -(nx - (float)n);
  const float p = 1.0f + r * (1.0f + r * (0.5f + r * (1.0f / 6.0f +
                  r * (1.0f / 24.0f + r * (1.0f / 120.0f + r * (1.0f / 720.0f))))));
  return exp_neg_table[n] * p;
}

/* GELU(x) = x/2 (1 + erf(x/sqrt2)) with erf by Abramowitz & Stegun 7.1.26
 * (cpp/include/hikoboshi/primitives/compute/gelu.hpp:22-51). */
static float erf_as(float v) {
  float sign = 1.0f;
  if (v < 0.0f) {
    sign = -1.0f;
    v = -v;
  }
  if (v > 4.0f) return sign;
  const float t = 1.0f / (1.0f + 0.3275911f * v);
  const float poly =
      (((((1.061405429f * t + -1.453152027f) * t) + 1.421413741f) * t +
        -0.284496736f) * t + 0.254829592f) * t;
  return sign * (1.0f - poly * exp_neg(-(v * v)));
}

static float gelu(float x) {
  return 0.5f * x * (1.0f + erf_as(x * 0.7071067811865475f));
}

/* Welford LayerNorm with population variance, eps 1e-5
 * (cpp/primitives/compute/layer_norm_scalar.cpp:8-40). */
static void layer_norm(const float* in, const float* g, const float* b,
                       float* out, int dim) {
  float mean = 0.0f, m2 = 0.0f;
  for (int d = 0; d < dim; ++d) {
    const float x = in[d];
    const float delta = x - mean;
    mean += delta / (float)(d + 1);
    m2 += delta * (x - mean);
  }
  const float inv_std = 1.0f / sqrtf(m2 / (float)dim + 1.0e-5f);
  for (int d = 0; d < dim; ++d) out[d] = (in[d] - mean) * inv_std * g[d] + b[d];
}

/* y[o] = sum_k x[k] W[o,k] (+ b[o]); W row-major [out, in]
 * (linear_nt_inline, cpp/include/hikoboshi/modules/mpnn/detail/
 * mpnn_inner_inline.hpp:312-343). */
static void linear(const float* x, const float* W, const float* b, int in,
                   int out, float* y) {
  for (int o = 0; o < out; ++o) {
    const float* w = W + (size_t)o * in;
    double acc = 0.0;
    for (int k = 0; k < in; ++k) acc += (double)x[k] * (double)w[k];
    y[o] = (float)acc + (b ? b[o] : 0.0f);
  }
}

/* ------------------------------------------------------------------------ */
/* Featurisation                                                            */
/* ------------------------------------------------------------------------ */

static int residue_present(const uint8_t* src, int r) {
  /* N, CA, C, O all non-missing (inverse_fold_scalar.cpp:82-88). */
  return src[r * 5 + 0] && src[r * 5 + 1] && src[r * 5 + 2] && src[r * 5 + 3];
}

static int kcount(int L) { return L < ORACLE_KMAX ? L : ORACLE_KMAX; }

static float sqdist_floor(const float* a, const float* b) {
  /* dx^2 + dy^2 + dz^2 + 1e-6, left to right, no contraction
   * (cpp/primitives/compute/knn_scalar.cpp:46-51). */
  const float dx = a[0] - b[0], dy = a[1] - b[1], dz = a[2] - b[2];
  return dx * dx + dy * dy + dz * dz + 1.0e-6f;
}

/* Top-K by (distance, index) with invalid pairs promoted to the row maximum
 * (cpp/primitives/compute/knn_scalar.cpp:72-168; configured as
 * inverse_fold_scalar.cpp:211-234). */
int oracle_knn(const float* coords, const uint8_t* src, int L, int32_t* idx,
               float* d2) {
  if (L <= 0) return 0;
  const int K = kcount(L);
  float* ca = (float*)malloc(sizeof(float) * 3 * (size_t)L);
  uint8_t* valid = (uint8_t*)malloc((size_t)L);
  for (int r = 0; r < L; ++r) {
    valid[r] = (uint8_t)residue_present(src, r);
    for (int x = 0; x < 3; ++x)
      ca[r * 3 + x] = src[r * 5 + 1] ? coords[(r * 5 + 1) * 3 + x] : 0.0f;
  }
  for (int q = 0; q < L; ++q) {
    int32_t* oi = idx + (size_t)q * K;
    float* od = d2 + (size_t)q * K;
    for (int s = 0; s < K; ++s) {
      oi[s] = -1;
      od[s] = INFINITY;
    }
    float rowmax = 1.0e-6f;
    if (valid[q])
      for (int t = 0; t < L; ++t)
        if (valid[t]) {
          const float c = sqdist_floor(ca + q * 3, ca + t * 3);
          if (c > rowmax) rowmax = c;
        }
    for (int t = 0; t < L; ++t) {
      const float dist = (valid[q] && valid[t]) ? sqdist_floor(ca + q * 3, ca + t * 3)
                                                : rowmax;
      int at = K;
      for (int s = 0; s < K; ++s)
        if (dist < od[s]) {
          at = s;
          break;
        }
      if (at == K) continue;
      for (int s = K - 1; s > at; --s) {
        od[s] = od[s - 1];
        oi[s] = oi[s - 1];
      }
      od[at] = dist;
      oi[at] = t;
    }
    for (int s = 0; s < K; ++s)
      if (od[s] == INFINITY) od[s] = rowmax;
  }
  free(ca);
  free(valid);
  return 0;
}

/* The 25 (query atom, neighbour atom) pairs in canonical slot numbers
 * N=0 CA=1 C=2 O=3 CB=4 (cpp/primitives/compute/atom_pair_distance_scalar.cpp:
 * 21-72). */
static const int kPairs[25][2] = {
    {1, 1}, {0, 0}, {2, 2}, {3, 3}, {4, 4}, {1, 0}, {1, 2}, {1, 3}, {1, 4},
    {0, 2}, {0, 3}, {0, 4}, {4, 2}, {4, 3}, {3, 2}, {0, 1}, {2, 1}, {3, 1},
    {4, 1}, {2, 0}, {3, 0}, {4, 0}, {2, 4}, {3, 4}, {2, 3}};

/* [16 positional | 25 x 16 RBF] per edge
 * (cpp/modules/mpnn/edge_rbf_features_scalar.cpp:45-152,
 *  cpp/primitives/compute/rbf_scalar.cpp:10-35). */
int oracle_edge_features(const oracle_weights* w, const float* coords,
                         const uint8_t* src, int L, const int32_t* idx,
                         float* feat) {
  exp_neg_init();
  const int K = kcount(L);
  const float* pw = w->t[ORACLE_T_POS_W];
  const float* pb = w->t[ORACLE_T_POS_B];
  const float sigma = (22.0f - 2.0f) / (16.0f / 0.7071067811865475f);
  const float two_s2 = 2.0f * sigma * sigma;
  const float step = (22.0f - 2.0f) / (float)(16 - 1);
  for (int i = 0; i < L; ++i)
    for (int k = 0; k < K; ++k) {
      float* row = feat + ((size_t)i * K + k) * EDGE_IN;
      const int j = idx[(size_t)i * K + k];
      if (j < 0 || j >= L) {
        memset(row, 0, sizeof(float) * EDGE_IN);
        continue;
      }
      int off = i - j;
      if (off < -32) off = -32;
      if (off > 32) off = 32;
      const int cls = off + 32;
      for (int d = 0; d < 16; ++d) row[d] = pw[d * 66 + cls] + pb[d];
      for (int p = 0; p < 25; ++p) {
        float* rb = row + 16 + p * 16;
        const int a = kPairs[p][0], b = kPairs[p][1];
        if (!src[i * 5 + a] || !src[j * 5 + b]) {
          memset(rb, 0, sizeof(float) * 16);
          continue;
        }
        float sq = 0.0f;
        for (int x = 0; x < 3; ++x) {
          const float delta = coords[(j * 5 + b) * 3 + x] - coords[(i * 5 + a) * 3 + x];
          sq += delta * delta;
        }
        const float dist = sqrtf(sq + 1.0e-6f);
        for (int f = 0; f < 16; ++f) {
          const float c = 2.0f + (float)f * step;
          const float dl = dist - c;
          rb[f] = exp_neg(-(dl * dl) / two_s2);
        }
      }
    }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Encoder (cpp/modules/mpnn/proteinmpnn_encoder_scalar.cpp:139-333 and     */
/* inverse_fold_scalar.cpp:236-352)                                          */
/* ------------------------------------------------------------------------ */

static void mlp3(const float* in, int in_dim, const float* const* t, float* out) {
  /* W1 -> GELU -> W2 -> GELU -> W3 with t = {W1.w,W1.b,W2.w,W2.b,W3.w,W3.b} */
  float a[H], b[H];
  linear(in, t[0], t[1], in_dim, H, a);
  for (int d = 0; d < H; ++d) a[d] = gelu(a[d]);
  linear(a, t[2], t[3], H, H, b);
  for (int d = 0; d < H; ++d) b[d] = gelu(b[d]);
  linear(b, t[4], t[5], H, H, out);
}

static void ffn_ln(float* h, const float* const* t_ffn, const float* g,
                   const float* bb) {
  /* h = LN(h + W_out GELU(W_in h + b_in) + b_out) */
  float f[FFN], o[H], s[H];
  linear(h, t_ffn[0], t_ffn[1], H, FFN, f);
  for (int d = 0; d < FFN; ++d) f[d] = gelu(f[d]);
  linear(f, t_ffn[2], t_ffn[3], FFN, H, o);
  for (int d = 0; d < H; ++d) s[d] = o[d] + h[d];
  layer_norm(s, g, bb, h, H);
}

int oracle_encode(const oracle_weights* w, const float* coords,
                  const uint8_t* src, int L, float* h_v, float* h_e,
                  int32_t* idx, float* mask, float* h_e0) {
  if (L <= 0) return 0;
  const int K = kcount(L);
  const size_t slots = (size_t)L * K;
  float* d2 = (float*)malloc(sizeof(float) * slots);
  float* feat = (float*)malloc(sizeof(float) * slots * EDGE_IN);
  for (int r = 0; r < L; ++r) mask[r] = residue_present(src, r) ? 1.0f : 0.0f;
  oracle_knn(coords, src, L, idx, d2);
  oracle_edge_features(w, coords, src, L, idx, feat);
  /* h_E0 = W_e LN(W_edge f) + b_e (inverse_fold_scalar.cpp:264-278) */
  for (size_t s = 0; s < slots; ++s) {
    float a[H], n[H];
    linear(feat + s * EDGE_IN, w->t[ORACLE_T_EDGE_W], NULL, EDGE_IN, H, a);
    layer_norm(a, w->t[ORACLE_T_NORM_E_W], w->t[ORACLE_T_NORM_E_B], n, H);
    linear(n, w->t[ORACLE_T_WE_W], w->t[ORACLE_T_WE_B], H, H, h_e + s * H);
  }
  if (h_e0) memcpy(h_e0, h_e, sizeof(float) * slots * H);
  memset(h_v, 0, sizeof(float) * (size_t)L * H);

  float* msg = (float*)malloc(sizeof(float) * slots * H);
  float* hnew = (float*)malloc(sizeof(float) * (size_t)L * H);
  float in[3 * H];
  for (int l = 0; l < 3; ++l) {
    const float* const* t = w->t + ORACLE_T_ENC0 + 22 * l;
    /* (1) messages from [h_i | e_ij | h_j] (:169-213) */
    for (int i = 0; i < L; ++i)
      for (int k = 0; k < K; ++k) {
        const size_t s = (size_t)i * K + k;
        const int j = idx[s];
        memcpy(in, h_v + (size_t)i * H, sizeof(float) * H);
        memcpy(in + H, h_e + s * H, sizeof(float) * H);
        if (j >= 0 && j < L) memcpy(in + 2 * H, h_v + (size_t)j * H, sizeof(float) * H);
        else memset(in + 2 * H, 0, sizeof(float) * H);
        mlp3(in, 3 * H, t + 0, msg + s * H);
      }
    /* (2) masked mean-free aggregation /30, residual LayerNorm (:215-249) */
    for (int i = 0; i < L; ++i) {
      float upd[H];
      memset(upd, 0, sizeof(upd));
      for (int k = 0; k < K; ++k) {
        const size_t s = (size_t)i * K + k;
        const int j = idx[s];
        if (j < 0 || j >= L) continue;
        const float alpha = (1.0f / 30.0f) * (mask[i] * mask[j]);
        if (alpha == 0.0f) continue;
        for (int d = 0; d < H; ++d) upd[d] += alpha * msg[s * H + d];
      }
      for (int d = 0; d < H; ++d) upd[d] += h_v[(size_t)i * H + d];
      layer_norm(upd, t[12], t[13], hnew + (size_t)i * H, H);
      /* (3) FFN + LayerNorm (:251-272), (4) mask (:274-287) */
      ffn_ln(hnew + (size_t)i * H, t + 18, t[14], t[15]);
      for (int d = 0; d < H; ++d) hnew[(size_t)i * H + d] *= mask[i];
    }
    memcpy(h_v, hnew, sizeof(float) * (size_t)L * H);
    /* (5) edge update with the updated nodes (:289-321) */
    for (int i = 0; i < L; ++i)
      for (int k = 0; k < K; ++k) {
        const size_t s = (size_t)i * K + k;
        const int j = idx[s];
        memcpy(in, h_v + (size_t)i * H, sizeof(float) * H);
        memcpy(in + H, h_e + s * H, sizeof(float) * H);
        if (j >= 0 && j < L) memcpy(in + 2 * H, h_v + (size_t)j * H, sizeof(float) * H);
        else memset(in + 2 * H, 0, sizeof(float) * H);
        mlp3(in, 3 * H, t + 6, msg + s * H);
      }
    for (size_t s = 0; s < slots; ++s) {
      const int j = idx[s];
      if (j < 0 || j >= L) continue;
      float sum[H];
      for (int d = 0; d < H; ++d) sum[d] = msg[s * H + d] + h_e[s * H + d];
      layer_norm(sum, t[16], t[17], h_e + s * H, H);
    }
  }
  free(msg);
  free(hnew);
  free(d2);
  free(feat);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Decoding order and RNG (cpp/modules/mpnn/decode_order_scalar.cpp,         */
/* sampler_scalar.cpp)                                                       */
/* ------------------------------------------------------------------------ */

static uint64_t splitmix64(uint64_t* s) {
  /* Steele/Lea/Flood SplitMix64 step (decode_order_scalar.cpp:21-27). */
  uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static double uniform01(uint64_t* s) {
  return (double)(splitmix64(s) >> 11) * (1.0 / 9007199254740992.0);
}

double oracle_uniform(uint64_t seed, int draw_index) {
  uint64_t s = seed;
  double u = 0.0;
  for (int i = 0; i <= draw_index; ++i) u = uniform01(&s);
  return u;
}

typedef struct {
  float score;
  int32_t index;
} order_key;

static int order_cmp(const void* a, const void* b) {
  const order_key* x = (const order_key*)a;
  const order_key* y = (const order_key*)b;
  if (x->score < y->score) return -1;
  if (x->score > y->score) return 1;
  return x->index < y->index ? -1 : (x->index > y->index ? 1 : 0);
}

/* Random order: ascending (mask+1e-4)*|BoxMuller|, ties by index
 * (decode_order_scalar.cpp:61-116). */
int oracle_decode_order(const float* mask, int L, uint64_t seed, int use_input,
                        const int32_t* input_order, int32_t* order) {
  if (use_input) {
    char* seen = (char*)calloc((size_t)(L > 0 ? L : 1), 1);
    for (int p = 0; p < L; ++p) {
      const int r = input_order ? input_order[p] : p;
      if (r < 0 || r >= L || seen[r]) {
        free(seen);
        return 1;
      }
      seen[r] = 1;
      order[p] = r;
    }
    free(seen);
    return 0;
  }
  order_key* keys = (order_key*)malloc(sizeof(order_key) * (size_t)(L > 0 ? L : 1));
  uint64_t s = seed;
  for (int r = 0; r < L; ++r) {
    double u1 = uniform01(&s);
    if (u1 <= 0.0) u1 = 1.0 / 9007199254740992.0;
    const double u2 = uniform01(&s);
    const double radius = sqrt(-2.0 * log(u1));
    const float z = (float)fabs(radius * cos(6.283185307179586476925286766559 * u2));
    const float cm = (mask ? mask[r] : 1.0f);
    keys[r].score = (cm + 0.0001f) * z;
    keys[r].index = r;
  }
  qsort(keys, (size_t)L, sizeof(order_key), order_cmp);
  for (int p = 0; p < L; ++p) order[p] = keys[p].index;
  free(keys);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Decoder layer (cpp/modules/mpnn/decoder_layer_scalar.cpp:26-151)          */
/* ------------------------------------------------------------------------ */

/* One DecLayer row: h (in/out) [H], ctx [K, 3H].  Attention mask null: every
 * slot counts with weight 1/30. */
static void dec_layer_row(const float* const* t, float* h, const float* ctx,
                          int K, float m) {
  float upd[H], in[4 * H], msg[H];
  memset(upd, 0, sizeof(upd));
  for (int k = 0; k < K; ++k) {
    memcpy(in, h, sizeof(float) * H);
    memcpy(in + H, ctx + (size_t)k * 3 * H, sizeof(float) * 3 * H);
    mlp3(in, 4 * H, t, msg);
    for (int d = 0; d < H; ++d) upd[d] += (1.0f / 30.0f) * msg[d];
  }
  for (int d = 0; d < H; ++d) upd[d] += h[d];
  layer_norm(upd, t[6], t[7], h, H);
  ffn_ln(h, t + 10, t[8], t[9]);
  if (m != 1.0f)
    for (int d = 0; d < H; ++d) h[d] *= m;
}

/* Context of slot k for row i at decoder layer l: bw*[h_E | h_S_j | h^l_j]
 * + fw*[h_E | 0 | h^enc_j] (inverse_fold_scalar.cpp:354-456, 665-728). */
static void build_ctx(const float* h_e, const int32_t* idx, int L, int K, int i,
                      const int32_t* pos, const float* mask, const float* hs,
                      const float* hl, const float* henc, float* ctx) {
  for (int k = 0; k < K; ++k) {
    const size_t s = (size_t)i * K + k;
    const int j = idx[s];
    float bw = 0.0f, fw = 0.0f;
    if (j >= 0 && j < L) {
      if (pos[j] < pos[i]) bw = mask[i];
      else fw = mask[i];
    }
    float* c = ctx + (size_t)k * 3 * H;
    for (int d = 0; d < H; ++d) c[d] = bw * h_e[s * H + d] + fw * h_e[s * H + d];
    for (int d = 0; d < H; ++d)
      c[H + d] = (j >= 0 && j < L) ? bw * hs[(size_t)j * H + d] : 0.0f;
    for (int d = 0; d < H; ++d)
      c[2 * H + d] = (j >= 0 && j < L)
                         ? bw * hl[(size_t)j * H + d] + fw * henc[(size_t)j * H + d]
                         : 0.0f;
  }
}

static void logits_row(const oracle_weights* w, const float* h, float* z) {
  linear(h, w->t[ORACLE_T_WOUT_W], w->t[ORACLE_T_WOUT_B], H, V, z);
}

static void log_softmax_row(const float* z, float T, float* out) {
  /* (z/T) - max - log sum exp  (log_softmax_scalar.cpp:8-37 for T = 1,
   * sampler_scalar.cpp:49-78 for the scaled form). */
  float zz[V], mx = -INFINITY, sum = 0.0f;
  for (int v = 0; v < V; ++v) {
    zz[v] = z[v] / T;
    if (zz[v] > mx) mx = zz[v];
  }
  for (int v = 0; v < V; ++v) sum += expf(zz[v] - mx);
  const float ls = logf(sum);
  for (int v = 0; v < V; ++v) out[v] = (zz[v] - mx) - ls;
}

static float sanitize_t(float T) { return (T > 0.0f && isfinite(T)) ? T : 1.0f; }

static float average_nll(const int32_t* tok, const float* lp, const float* mask,
                         int L) {
  /* inverse_fold_scalar.cpp:471-493 */
  double loss = 0.0, cnt = 0.0;
  for (int r = 0; r < L; ++r) {
    if (mask[r] == 0.0f) continue;
    if (tok[r] < 0 || tok[r] >= V) continue;
    loss -= (double)lp[(size_t)r * V + tok[r]];
    cnt += (double)mask[r];
  }
  return cnt > 0.0 ? (float)(loss / cnt) : 0.0f;
}

/* Parallel causal pass over all rows (inverse_fold_scalar.cpp:575-663). */
static int teacher_forced_impl(const oracle_weights* w, const float* coords,
                               const uint8_t* src, int L, const int32_t* tokens,
                               const int32_t* order, float T, float* log_probs) {
  const int K = kcount(L);
  const size_t slots = (size_t)L * K;
  float* hv = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* he = (float*)malloc(sizeof(float) * slots * H);
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * slots);
  float* mask = (float*)malloc(sizeof(float) * (size_t)L);
  oracle_encode(w, coords, src, L, hv, he, idx, mask, NULL);
  int32_t* pos = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
  for (int p = 0; p < L; ++p) pos[order[p]] = p;
  float* hs = (float*)malloc(sizeof(float) * (size_t)L * H);
  for (int r = 0; r < L; ++r)
    memcpy(hs + (size_t)r * H, w->t[ORACLE_T_WS] + (size_t)tokens[r] * H,
           sizeof(float) * H);
  float* hl = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* hn = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* ctx = (float*)malloc(sizeof(float) * (size_t)K * 3 * H);
  memcpy(hl, hv, sizeof(float) * (size_t)L * H);
  for (int l = 0; l < 3; ++l) {
    const float* const* t = w->t + ORACLE_T_DEC0 + 14 * l;
    for (int i = 0; i < L; ++i) {
      build_ctx(he, idx, L, K, i, pos, mask, hs, hl, hv, ctx);
      memcpy(hn + (size_t)i * H, hl + (size_t)i * H, sizeof(float) * H);
      dec_layer_row(t, hn + (size_t)i * H, ctx, K, mask[i]);
    }
    memcpy(hl, hn, sizeof(float) * (size_t)L * H);
  }
  for (int i = 0; i < L; ++i) {
    float z[V];
    logits_row(w, hl + (size_t)i * H, z);
    log_softmax_row(z, T, log_probs + (size_t)i * V);
  }
  free(hv); free(he); free(idx); free(mask); free(pos); free(hs); free(hl);
  free(hn); free(ctx);
  return 0;
}

static int validate_tokens(const int32_t* tokens, int L) {
  for (int r = 0; r < L; ++r)
    if (tokens[r] < 0 || tokens[r] >= V) return 1;
  return 0;
}

int oracle_teacher_forced(const oracle_weights* w, const float* coords,
                          const uint8_t* src, int L, const int32_t* tokens,
                          const int32_t* order_in, uint64_t seed,
                          float* log_probs, int32_t* order_out, float* score) {
  if (L <= 0) return 0;
  if (validate_tokens(tokens, L)) return 1;
  float* mask = (float*)malloc(sizeof(float) * (size_t)L);
  for (int r = 0; r < L; ++r) mask[r] = residue_present(src, r) ? 1.0f : 0.0f;
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
  int st = oracle_decode_order(mask, L, seed, order_in != NULL, order_in, order);
  if (st == 0) {
    teacher_forced_impl(w, coords, src, L, tokens, order, 1.0f, log_probs);
    if (order_out) memcpy(order_out, order, sizeof(int32_t) * (size_t)L);
    if (score) *score = average_nll(tokens, log_probs, mask, L);
  }
  free(mask);
  free(order);
  return st;
}

int oracle_teacher_forced_scaled(const oracle_weights* w, const float* coords,
                                 const uint8_t* src, int L,
                                 const int32_t* tokens, const int32_t* order,
                                 float temperature, float* log_probs) {
  if (L <= 0) return 0;
  if (validate_tokens(tokens, L)) return 1;
  return teacher_forced_impl(w, coords, src, L, tokens, order,
                             sanitize_t(temperature), log_probs);
}

/* Autoregressive design (inverse_fold_scalar.cpp:752-888, sampler_scalar.cpp:
 * 49-131). */
int oracle_inverse_fold(const oracle_weights* w, const float* coords,
                        const uint8_t* src, int L, uint64_t seed,
                        float temperature, int n_to_c, const int32_t* order_in,
                        int32_t* tokens, float* log_probs, int32_t* order_out,
                        float* score) {
  if (L <= 0) return 0;
  if (!(isfinite(temperature)) || temperature < 0.0f) return 1;
  const int K = kcount(L);
  const size_t slots = (size_t)L * K;
  float* hv = (float*)malloc(sizeof(float) * (size_t)L * H);
  float* he = (float*)malloc(sizeof(float) * slots * H);
  int32_t* idx = (int32_t*)malloc(sizeof(int32_t) * slots);
  float* mask = (float*)malloc(sizeof(float) * (size_t)L);
  oracle_encode(w, coords, src, L, hv, he, idx, mask, NULL);
  int32_t* order = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
  int identity = n_to_c || order_in != NULL;
  int st = oracle_decode_order(mask, L, seed, identity, order_in, order);
  if (st != 0) {
    free(hv); free(he); free(idx); free(mask); free(order);
    return st;
  }
  int32_t* pos = (int32_t*)malloc(sizeof(int32_t) * (size_t)L);
  for (int p = 0; p < L; ++p) pos[order[p]] = p;
  /* h_V stack [4, L, H]: layer 0 = encoder output, others start at zero. */
  float* stack = (float*)calloc((size_t)4 * L * H, sizeof(float));
  memcpy(stack, hv, sizeof(float) * (size_t)L * H);
  float* hs = (float*)calloc((size_t)L * H, sizeof(float));
  float* ctx = (float*)malloc(sizeof(float) * (size_t)K * 3 * H);
  const int greedy = temperature <= 0.0f;
  const float T = sanitize_t(temperature);
  uint64_t rng = seed;
  for (int p = 0; p < L; ++p) {
    const int t = order[p];
    if (mask[t] == 0.0f) {
      tokens[t] = V - 1;
      memset(log_probs + (size_t)t * V, 0, sizeof(float) * V);
      memcpy(hs + (size_t)t * H, w->t[ORACLE_T_WS] + (size_t)(V - 1) * H,
             sizeof(float) * H);
      continue;
    }
    float h[H];
    for (int l = 0; l < 3; ++l) {
      const float* hl = stack + (size_t)l * L * H;
      build_ctx(he, idx, L, K, t, pos, mask, hs, hl, hv, ctx);
      memcpy(h, hl + (size_t)t * H, sizeof(float) * H);
      dec_layer_row(w->t + ORACLE_T_DEC0 + 14 * l, h, ctx, K, mask[t]);
      memcpy(stack + (size_t)(l + 1) * L * H + (size_t)t * H, h, sizeof(float) * H);
    }
    float z[V], lp[V], prob[V], zz[V], mx = -INFINITY, sum = 0.0f;
    logits_row(w, h, z);
    for (int v = 0; v < V; ++v) {
      zz[v] = z[v] / T;
      if (zz[v] > mx) mx = zz[v];
    }
    for (int v = 0; v < V; ++v) {
      prob[v] = expf(zz[v] - mx);
      sum += prob[v];
    }
    const float ls = logf(sum), inv = 1.0f / sum;
    for (int v = 0; v < V; ++v) {
      prob[v] *= inv;
      lp[v] = (zz[v] - mx) - ls;
    }
    int tok = V - 1;
    if (greedy) {
      tok = 0;
      for (int v = 1; v < V; ++v)
        if (zz[v] > zz[tok]) tok = v;
    } else {
      const double u = uniform01(&rng);
      double cum = 0.0;
      for (int v = 0; v < V; ++v) {
        cum += (double)prob[v];
        if (u < cum) {
          tok = v;
          break;
        }
      }
    }
    tokens[t] = tok;
    memcpy(log_probs + (size_t)t * V, lp, sizeof(float) * V);
    memcpy(hs + (size_t)t * H, w->t[ORACLE_T_WS] + (size_t)tok * H, sizeof(float) * H);
  }
  if (order_out) memcpy(order_out, order, sizeof(int32_t) * (size_t)L);
  if (score) *score = average_nll(tokens, log_probs, mask, L);
  free(hv); free(he); free(idx); free(mask); free(order); free(pos); free(stack);
  free(hs); free(ctx);
  return 0;
}
