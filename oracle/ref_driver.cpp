// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// Thin C-ABI shim around the *reference's own* CPU implementation of the
// ProteinMPNN v_48_020 design path, compiled from the reference sources where
// they lie (see oracle/Makefile).  It lets the test-suite and the bench's
// reference arm call, from Python via ctypes:
//
//   ref_load_weights        binds the 118 fp32 safetensors tensors into the
//                           reference's ProteinMpnnV48020Weights borrowed view
//                           (names map 1:1, cpp/include/hikoboshi/universal/
//                           detail/proteinmpnn_v48_020_schema.hpp:127-160)
//   ref_knn                 primitives::compute::knn_scalar, configured exactly
//                           as build_knn does (modules/mpnn/inverse_fold_scalar
//                           .cpp:211-234)
//   ref_teacher_forced      modules::mpnn::proteinmpnn_teacher_forced_forward_
//                           scalar (inverse_fold_scalar.cpp:905-952)
//   ref_inverse_fold        modules::mpnn::proteinmpnn_inverse_fold_scalar with
//                           the options algorithms/inverse_fold.cpp:304-310 sets
//   ref_design              algorithms::inverse_fold_proteinmpnn_v48_020
//                           (algorithms/inverse_fold.cpp:221-356): the repo's
//                           `design` path minus file IO
//   ref_decode_order        modules::mpnn::proteinmpnn_decode_order_scalar
//   ref_design_noisy        ref_design with backbone_noise > 0
//
// The workspace holders below only size plain std::vectors with the
// reference's own plan-count helpers; all arithmetic is the reference's.

#include <hikoboshi/algorithms/inverse_fold.hpp>
#include <hikoboshi/modules/detail/mpnn_workspace.hpp>
#include <hikoboshi/modules/mpnn/inverse_fold.hpp>
#include <hikoboshi/modules/mpnn/proteinmpnn_decoder.hpp>
#include <hikoboshi/primitives/compute/knn.hpp>
#include <hikoboshi/universal/detail/proteinmpnn_v48_020_weights.hpp>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

namespace hd = hikoboshi::modules::detail;
namespace hm = hikoboshi::modules::mpnn;
namespace hu = hikoboshi::universal;
namespace pmp = hikoboshi::universal::detail;

constexpr std::size_t kH = pmp::kProteinMpnnV48020Hidden;
constexpr std::size_t kV = pmp::kProteinMpnnV48020Vocab;

struct TensorRec {
  std::vector<std::size_t> shape;
  const float* data = nullptr;
  std::size_t count = 0;
};

std::vector<unsigned char> g_blob;
std::map<std::string, TensorRec> g_tensors;
pmp::ProteinMpnnV48020Weights g_weights{};
bool g_loaded = false;

// Minimal scanner for the safetensors JSON header: {"name":{"dtype":"F32",
// "shape":[a,b],"data_offsets":[s,e]},...}.  Only what the F32 weight file
// uses is understood.
bool parse_header(const std::string& h, std::size_t data_base) {
  std::size_t pos = 0;
  while (true) {
    std::size_t q0 = h.find('"', pos);
    if (q0 == std::string::npos) break;
    std::size_t q1 = h.find('"', q0 + 1);
    std::string name = h.substr(q0 + 1, q1 - q0 - 1);
    std::size_t obj0 = h.find('{', q1);
    std::size_t obj1 = h.find('}', obj0);
    if (obj0 == std::string::npos || obj1 == std::string::npos) break;
    std::string body = h.substr(obj0, obj1 - obj0 + 1);
    pos = obj1 + 1;
    if (name == "__metadata__") continue;
    if (body.find("\"F32\"") == std::string::npos) return false;
    TensorRec rec;
    std::size_t sp = body.find("\"shape\"");
    std::size_t sb = body.find('[', sp), se = body.find(']', sb);
    std::string dims = body.substr(sb + 1, se - sb - 1);
    std::size_t count = 1;
    char* cur = dims.data();
    while (*cur) {
      char* end = nullptr;
      unsigned long v = std::strtoul(cur, &end, 10);
      if (end == cur) { ++cur; continue; }
      rec.shape.push_back(v);
      count *= v;
      cur = end;
    }
    std::size_t op = body.find("\"data_offsets\"");
    std::size_t ob = body.find('[', op);
    char* end = nullptr;
    unsigned long s = std::strtoul(body.c_str() + ob + 1, &end, 10);
    unsigned long e = std::strtoul(end + 1, nullptr, 10);
    if ((e - s) != count * sizeof(float)) return false;
    rec.data = reinterpret_cast<const float*>(g_blob.data() + data_base + s);
    rec.count = count;
    g_tensors[name] = rec;
  }
  return true;
}

hu::Span<const float> span_of(const std::string& name, bool* ok) {
  auto it = g_tensors.find(name);
  if (it == g_tensors.end()) {
    std::fprintf(stderr, "ref_driver: missing tensor %s\n", name.c_str());
    *ok = false;
    return {nullptr, 0};
  }
  return {it->second.data, it->second.count};
}

void bind_linear(pmp::ProteinMpnnV48020LinearWeights& w, const std::string& p,
                 bool* ok) {
  w.weight = span_of(p + ".weight", ok);
  w.bias = span_of(p + ".bias", ok);
}

void bind_norm(pmp::ProteinMpnnV48020NormWeights& w, const std::string& p,
               bool* ok) {
  w.weight = span_of(p + ".weight", ok);
  w.bias = span_of(p + ".bias", ok);
}

struct EncoderStore {
  explicit EncoderStore(std::size_t L, std::size_t K)
      : plan{L, kH, K, pmp::kProteinMpnnV48020RbfCount,
             pmp::kProteinMpnnV48020NumEncoderLayers},
        ca(hd::mpnn64_ca_coordinate_count(plan)),
        feat(std::max(hd::mpnn64_residue_feature_count(plan),
                      hd::mpnn64_neighbor_slot_count(plan) * 3U * kH)),
        idx(hd::mpnn64_neighbor_slot_count(plan)),
        d2(hd::mpnn64_neighbor_slot_count(plan)),
        rbf(hd::mpnn64_neighbor_rbf_count(plan)),
        rs(hd::mpnn64_residue_hidden_count(plan)),
        gs(hd::mpnn64_neighbor_hidden_count(plan)),
        es(hd::mpnn64_neighbor_hidden_count(plan)),
        ms(hd::mpnn64_neighbor_hidden_count(plan)),
        pms(hd::mpnn64_neighbor_hidden_count(plan)),
        scr(hd::mpnn64_residue_hidden_count(plan)),
        ffn(hd::mpnn64_ffn_hidden_count(plan)) {}
  template <typename T>
  static hu::Span<T> sp(std::vector<T>& v) {
    return {v.empty() ? nullptr : v.data(), v.size()};
  }
  hd::Mpnn64Workspace view() {
    return {plan, sp(ca), sp(feat), sp(idx), sp(d2), sp(rbf), sp(rs),
            sp(gs), sp(es), sp(ms), sp(pms), sp(scr), sp(ffn)};
  }
  hd::Mpnn64MemoryPlan plan;
  std::vector<float> ca, feat;
  std::vector<std::int32_t> idx;
  std::vector<float> d2, rbf, rs, gs, es, ms, pms, scr, ffn;
};

struct DecoderStore {
  explicit DecoderStore(std::size_t L, std::size_t K)
      : plan{std::max<std::size_t>(L, 1U), kH, K,
             pmp::kProteinMpnnV48020DecoderNumInDimension,
             pmp::kProteinMpnnV48020FfnHidden},
        mi(hm::proteinmpnn_decoder_message_input_count(plan)),
        ms(hm::proteinmpnn_decoder_neighbor_hidden_count(plan)),
        pms(hm::proteinmpnn_decoder_neighbor_hidden_count(plan)),
        scr(hm::proteinmpnn_decoder_residue_hidden_count(plan)),
        ffn(hm::proteinmpnn_decoder_ffn_hidden_count(plan)) {}
  hm::ProteinMpnnDecoderWorkspace view() {
    return {plan, EncoderStore::sp(mi), EncoderStore::sp(ms),
            EncoderStore::sp(pms), EncoderStore::sp(scr),
            EncoderStore::sp(ffn)};
  }
  hm::ProteinMpnnDecoderMemoryPlan plan;
  std::vector<float> mi, ms, pms, scr, ffn;
};

}  // namespace

extern "C" {

// Returns 0 on success.
int ref_load_weights(const char* path) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return 1;
  std::fseek(f, 0, SEEK_END);
  long n = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  g_blob.resize(static_cast<std::size_t>(n));
  if (std::fread(g_blob.data(), 1, g_blob.size(), f) != g_blob.size()) {
    std::fclose(f);
    return 2;
  }
  std::fclose(f);
  std::uint64_t hlen = 0;
  std::memcpy(&hlen, g_blob.data(), 8);
  std::string header(reinterpret_cast<const char*>(g_blob.data() + 8), hlen);
  g_tensors.clear();
  if (!parse_header(header, 8 + hlen)) return 3;
  bool ok = true;
  auto& w = g_weights;
  bind_linear(w.features.embeddings.linear, "features.embeddings.linear", &ok);
  w.features.edge_embedding.weight =
      span_of("features.edge_embedding.weight", &ok);
  bind_norm(w.features.norm_edges, "features.norm_edges", &ok);
  bind_linear(w.W_e, "W_e", &ok);
  w.W_s.weight = span_of("W_s.weight", &ok);
  for (int l = 0; l < 3; ++l) {
    const std::string p = "encoder_layers." + std::to_string(l) + ".";
    auto& e = w.encoder_layers[l];
    bind_linear(e.W1, p + "W1", &ok);
    bind_linear(e.W2, p + "W2", &ok);
    bind_linear(e.W3, p + "W3", &ok);
    bind_linear(e.W11, p + "W11", &ok);
    bind_linear(e.W12, p + "W12", &ok);
    bind_linear(e.W13, p + "W13", &ok);
    bind_norm(e.norm1, p + "norm1", &ok);
    bind_norm(e.norm2, p + "norm2", &ok);
    bind_norm(e.norm3, p + "norm3", &ok);
    bind_linear(e.dense.W_in, p + "dense.W_in", &ok);
    bind_linear(e.dense.W_out, p + "dense.W_out", &ok);
  }
  for (int l = 0; l < 3; ++l) {
    const std::string p = "decoder_layers." + std::to_string(l) + ".";
    auto& d = w.decoder_layers[l];
    bind_linear(d.W1, p + "W1", &ok);
    bind_linear(d.W2, p + "W2", &ok);
    bind_linear(d.W3, p + "W3", &ok);
    bind_norm(d.norm1, p + "norm1", &ok);
    bind_norm(d.norm2, p + "norm2", &ok);
    bind_linear(d.dense.W_in, p + "dense.W_in", &ok);
    bind_linear(d.dense.W_out, p + "dense.W_out", &ok);
  }
  bind_linear(w.W_out, "W_out", &ok);
  g_loaded = ok && g_tensors.size() == 118;
  return g_loaded ? 0 : 4;
}

// CA kNN exactly as build_knn configures it (include_self, validity = N/CA/C/O
// all present, CA of a residue with missing CA read as zero).
int ref_knn(const float* coords, const std::uint8_t* sources, std::size_t L,
            std::int32_t* out_idx, float* out_d2) {
  const std::size_t K = hm::proteinmpnn_v48_020_effective_neighbor_count(L);
  std::vector<float> ca(L * 3, 0.0F);
  std::vector<std::uint8_t> valid(L, 0);
  for (std::size_t r = 0; r < L; ++r) {
    bool present = true;
    for (int a = 0; a < 4; ++a) present = present && sources[r * 5 + a] != 0;
    valid[r] = present ? 1 : 0;
    const bool ca_present = sources[r * 5 + 1] != 0;
    for (int x = 0; x < 3; ++x)
      ca[r * 3 + x] = ca_present ? coords[(r * 5 + 1) * 3 + x] : 0.0F;
  }
  hikoboshi::primitives::compute::KnnScalarRequest req{};
  req.query_coordinates = ca.data();
  req.target_coordinates = ca.data();
  req.query_validity_mask = valid.data();
  req.target_validity_mask = valid.data();
  req.query_count = L;
  req.target_count = L;
  req.k = K;
  req.include_self = true;
  req.treat_zero_coords_as_invalid = false;
  hikoboshi::primitives::compute::KnnScalarOutput out{};
  out.neighbor_indices = out_idx;
  out.neighbor_squared_distances = out_d2;
  hikoboshi::primitives::compute::knn_scalar(req, out);
  return 0;
}

int ref_decode_order(const float* residue_mask, std::size_t L,
                     std::uint64_t seed, int use_input,
                     const std::int32_t* input_order, std::int32_t* out) {
  hm::ProteinMpnnDecodeOrderRequest req{};
  req.chain_mask = nullptr;
  req.residue_mask = residue_mask;
  req.input_order = input_order;
  req.residue_count = L;
  req.seed = seed;
  req.use_input_decoding_order = use_input != 0;
  hm::ProteinMpnnDecodeOrderOutput o{};
  o.decoding_order = out;
  o.order_scores = nullptr;
  return static_cast<int>(hm::proteinmpnn_decode_order_scalar(req, o).code);
}

int ref_teacher_forced(const float* coords, const std::uint8_t* sources,
                       std::size_t L, const std::int32_t* tokens,
                       const std::int32_t* input_order, std::uint64_t seed,
                       float* log_probs, std::int32_t* order_out,
                       float* score) {
  if (!g_loaded) return 100;
  const std::size_t K = hm::proteinmpnn_v48_020_effective_neighbor_count(L);
  EncoderStore es(L, K);
  DecoderStore ds(L, K);
  hd::Mpnn64Workspace ew = es.view();
  hm::ProteinMpnnDecoderWorkspace dw = ds.view();
  hm::ProteinMpnnInverseFoldOptions opt{};
  opt.seed = seed;
  opt.decode_order_seed = seed;
  opt.use_input_decoding_order = input_order != nullptr;
  hm::ProteinMpnnTeacherForcedRequest req{};
  req.coordinates = coords;
  req.atom_sources = reinterpret_cast<const hu::AtomSource*>(sources);
  req.token_ids = tokens;
  req.weights = &g_weights;
  req.encoder_workspace = &ew;
  req.decoder_workspace = &dw;
  req.residue_count = L;
  req.input_decoding_order = input_order;
  req.options = opt;
  hm::ProteinMpnnTeacherForcedOutput out{};
  out.log_probs = log_probs;
  out.decoding_order = order_out;
  out.sequence_score = score;
  out.residue_count = L;
  out.vocab_size = kV;
  return static_cast<int>(
      hm::proteinmpnn_teacher_forced_forward_scalar(req, out).code);
}

int ref_inverse_fold(const float* coords, const std::uint8_t* sources,
                     std::size_t L, std::uint64_t seed, float temperature,
                     int n_to_c, std::int32_t* tokens, float* log_probs,
                     std::int32_t* order_out, float* score) {
  if (!g_loaded) return 100;
  const std::size_t K = hm::proteinmpnn_v48_020_effective_neighbor_count(L);
  EncoderStore es(L, K);
  DecoderStore ds(L, K);
  hd::Mpnn64Workspace ew = es.view();
  hm::ProteinMpnnDecoderWorkspace dw = ds.view();
  std::vector<std::int32_t> identity(L);
  for (std::size_t i = 0; i < L; ++i) identity[i] = static_cast<int>(i);
  hm::ProteinMpnnInverseFoldOptions opt{};
  opt.seed = seed;
  opt.decode_order_seed = seed;
  opt.temperature = temperature;
  opt.greedy = temperature <= 0.0F;
  opt.use_input_decoding_order = n_to_c != 0;
  hm::ProteinMpnnInverseFoldRequest req{};
  req.coordinates = coords;
  req.atom_sources = reinterpret_cast<const hu::AtomSource*>(sources);
  req.weights = &g_weights;
  req.encoder_workspace = &ew;
  req.decoder_workspace = &dw;
  req.residue_count = L;
  req.input_decoding_order = n_to_c ? identity.data() : nullptr;
  req.options = opt;
  std::vector<char> seq(L + 1, '\0');
  hm::ProteinMpnnInverseFoldOutput out{};
  out.token_ids = tokens;
  out.sequence = seq.data();
  out.log_probs = log_probs;
  out.decoding_order = order_out;
  out.sequence_score = score;
  out.residue_count = L;
  out.vocab_size = kV;
  return static_cast<int>(hm::proteinmpnn_inverse_fold_scalar(req, out).code);
}

// The algorithms-layer design call: num_seqs sequences with seed+index,
// decode_order 0 = random, 1 = n_to_c.  Outputs are [num_seqs, L] tokens
// (as alphabet indices), [num_seqs, L, 21] log-probs, [num_seqs] scores.
int ref_design_noisy(const float* coords, const std::uint8_t* sources,
                     std::size_t L, std::size_t num_seqs, std::uint64_t seed,
                     float temperature, int decode_order, float backbone_noise,
                     std::int32_t* tokens, float* log_probs, float* scores);

int ref_design(const float* coords, const std::uint8_t* sources,
               std::size_t L, std::size_t num_seqs, std::uint64_t seed,
               float temperature, int decode_order, std::int32_t* tokens,
               float* log_probs, float* scores) {
  return ref_design_noisy(coords, sources, L, num_seqs, seed, temperature, decode_order, 0.0f,
                          tokens, log_probs, scores);
}

// ref_design with the algorithm layer's backbone_noise option
// (algorithms/inverse_fold.cpp:191-207, 296-302).
int ref_design_noisy(const float* coords, const std::uint8_t* sources,
                     std::size_t L, std::size_t num_seqs, std::uint64_t seed,
                     float temperature, int decode_order, float backbone_noise,
                     std::int32_t* tokens, float* log_probs, float* scores) {
  if (!g_loaded) return 100;
  hikoboshi::algorithms::InverseFoldRequest req{};
  req.structure.residue_count = L;
  req.structure.coordinates = {coords, L * 15};
  req.structure.atom_sources = {reinterpret_cast<const hu::AtomSource*>(sources),
                                L * 5};
  req.structure.residue_codes = {nullptr, 0};
  req.structure.residues = {nullptr, 0};
  req.weights = &g_weights;
  req.options.sampling_temp = temperature;
  req.options.num_seqs = num_seqs;
  req.options.seed = seed;
  req.options.decode_order =
      decode_order == 1 ? hikoboshi::algorithms::InverseFoldDecodeOrder::NToC
                        : hikoboshi::algorithms::InverseFoldDecodeOrder::Random;
  req.options.keep_log_probs = log_probs != nullptr;
  req.options.backbone_noise = backbone_noise;
  auto res = hikoboshi::algorithms::inverse_fold_proteinmpnn_v48_020(req);
  if (!res.status.ok()) return static_cast<int>(res.status.code);
  static const char kAlpha[] = "ACDEFGHIKLMNPQRSTVWYX";
  for (std::size_t s = 0; s < num_seqs; ++s) {
    const std::string& q = res.value.sequences[s].sequence;
    for (std::size_t i = 0; i < L; ++i) {
      const char* hit = std::strchr(kAlpha, q[i]);
      tokens[s * L + i] = hit ? static_cast<std::int32_t>(hit - kAlpha) : 20;
    }
    if (scores) scores[s] = static_cast<float>(res.value.sequences[s].score);
  }
  if (log_probs) {
    std::memcpy(log_probs, res.value.logprobs.values.data(),
                num_seqs * L * kV * sizeof(float));
  }
  return 0;
}

}  // extern "C"
