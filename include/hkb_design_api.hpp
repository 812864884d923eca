// C++17 adapter over the C ABI with the reference's request / result types
// for the design path, so C++ callers of hikoboshi::api::Engine::inverse_fold
// and the hikoboshi::io structure / writer functions switch by changing the
// include (cpp/include/hikoboshi/api/engine.hpp, api/results.hpp,
// io/structure_loader.hpp, io/design_fasta_writer.hpp).  Header-only: every
// function forwards to libhkb_mpnn.so.
#pragma once

#include <cmath>
#include <cstdint>
#include <fstream>
#include <memory>
#include <optional>
#include <sstream>
#include <string>
#include <string_view>
#include <vector>

#include "hkb_mpnn.h"

namespace hikoboshi {

namespace universal {
using Status = hkb_status;   // {code, static detail}; codes as universal::StatusCode
template <typename T>
struct Result {
  Status status{HKB_OK, ""};
  T value{};
};
inline bool ok(const Status& s) { return s.code == HKB_OK; }
}  // namespace universal

namespace io {

// io::LoadedStructure: owns one normalised chain.
class LoadedStructure {
 public:
  int32_t residue_count() const { return h_ ? hkb_structure_residue_count(h_.get()) : 0; }
  const std::vector<float>& coordinates() const { return coords_; }
  const std::vector<uint8_t>& atom_sources() const { return sources_; }
  const std::string& residue_codes() const { return codes_; }
  static universal::Result<LoadedStructure> adopt(hkb_structure* h) {
    universal::Result<LoadedStructure> r;
    r.value.h_ = std::shared_ptr<hkb_structure>(h, Del{});
    const int32_t L = hkb_structure_residue_count(h);
    r.value.coords_.resize((size_t)L * 15);
    r.value.sources_.resize((size_t)L * 5);
    r.value.codes_.resize((size_t)L);
    r.status = hkb_structure_copy(h, r.value.coords_.data(), r.value.sources_.data(),
                                  r.value.codes_.data());
    return r;
  }

 private:
  struct Del {
    void operator()(hkb_structure* p) const { hkb_structure_destroy(p); }
  };
  std::shared_ptr<hkb_structure> h_{nullptr, Del{}};
  std::vector<float> coords_;
  std::vector<uint8_t> sources_;
  std::string codes_;
};

inline universal::Result<LoadedStructure> load_structure_from_file(
    std::string_view path, const hkb_structure_options* options = nullptr) {
  hkb_structure* h = nullptr;
  const std::string p(path);
  const hkb_status st = hkb_structure_load_file(p.c_str(), options, &h);
  if (st.code != HKB_OK) return {st, {}};
  return LoadedStructure::adopt(h);
}

}  // namespace io

namespace api {

enum class InverseFoldDecodeOrder { Random, NToC };

// A structure view: canonical [L,5,3] coordinates and [L,5] atom sources
// (residue codes optional, for recovery_vs_native).
struct StructureView {
  size_t residue_count = 0;
  const float* coordinates = nullptr;
  const uint8_t* atom_sources = nullptr;
  const char* residue_codes = nullptr;
};

struct InverseFoldRequest {
  StructureView structure{};
  std::string pdb_path;
  std::string package = "proteinmpnn-v48-eps020";
  float sampling_temp = 0.1f;
  size_t num_seqs = 1;
  uint64_t seed = 0;
  InverseFoldDecodeOrder decode_order = InverseFoldDecodeOrder::Random;
  float backbone_noise = 0.0f;
  std::string logprobs_out;   // non-empty: keep the [N,L,21] log-probs
};

struct InverseFoldSequenceResult {
  std::string sequence;
  double score = 0.0;
  std::optional<double> recovery_vs_native;
  uint64_t seed = 0;
  InverseFoldDecodeOrder decode_order = InverseFoldDecodeOrder::Random;
};

struct InverseFoldLogProbsArtifact {
  std::string path;
  size_t num_seqs = 0, residue_count = 0, vocab_size = 0;
  std::vector<float> values;   // [num_seqs, residue_count, vocab_size]
};

struct InverseFoldResult {
  std::vector<InverseFoldSequenceResult> sequences;
  InverseFoldLogProbsArtifact logprobs{};
};

// One engine per device; precision HKB_PRECISION_FP32 reproduces the
// reference's arithmetic, HKB_PRECISION_F16 is the tensor-core mode.
class Engine {
 public:
  static universal::Result<Engine> create(const std::string& weights_path, int device = 0,
                                          int32_t precision = HKB_PRECISION_FP32) {
    universal::Result<Engine> r;
    std::ifstream f(weights_path, std::ios::binary);
    if (!f) return {{HKB_UNAVAILABLE, "ProteinMPNN weights file not readable"}, {}};
    std::ostringstream b;
    b << f.rdbuf();
    const std::string blob = b.str();
    hkb_engine* e = nullptr;
    r.status = hkb_mpnn_create(blob.data(), blob.size(), device, precision, &e);
    if (r.status.code == HKB_OK) r.value.e_.reset(e, hkb_mpnn_destroy);
    return r;
  }

  // algorithms::inverse_fold_proteinmpnn_v48_020 semantics
  // (algorithms/inverse_fold.cpp:221-356) on the device engine.
  universal::Result<InverseFoldResult> inverse_fold(const InverseFoldRequest& rq) const;

  hkb_engine* handle() const { return e_.get(); }

 private:
  std::shared_ptr<hkb_engine> e_;
};

inline universal::Result<InverseFoldResult> Engine::inverse_fold(
    const InverseFoldRequest& rq) const {
  universal::Result<InverseFoldResult> r;
  const StructureView& s = rq.structure;
  const int32_t L = static_cast<int32_t>(s.residue_count);
  if (!e_) return {{HKB_FAILED_PRECONDITION, "ProteinMPNN inverse-folding weights are not available"}, {}};
  if (L == 0) return {{HKB_INVALID_ARGUMENT, "inverse-fold structure must contain at least one residue"}, {}};
  if (!s.coordinates || !s.atom_sources)
    return {{HKB_INVALID_ARGUMENT, "inverse-fold structure must provide canonical backbone atoms"}, {}};
  if (rq.num_seqs == 0) return {{HKB_INVALID_ARGUMENT, "inverse-fold num_seqs must be greater than zero"}, {}};
  if (!std::isfinite(rq.sampling_temp) || rq.sampling_temp < 0.0f)
    return {{HKB_INVALID_ARGUMENT, "inverse-fold sampling_temp must be finite and >= 0"}, {}};
  if (!std::isfinite(rq.backbone_noise) || rq.backbone_noise < 0.0f)
    return {{HKB_INVALID_ARGUMENT, "inverse-fold backbone_noise must be finite and >= 0"}, {}};
  const size_t N = rq.num_seqs;
  const bool noisy = rq.backbone_noise > 0.0f;
  // noise: each sequence its own noisy copy, i.e. its own batch entry
  const int32_t B = noisy ? static_cast<int32_t>(N) : 1;
  std::vector<float> coords((size_t)B * L * 15);
  std::vector<uint8_t> src((size_t)B * L * 5);
  std::vector<int32_t> lens(B, L), nseq(B, noisy ? 1 : static_cast<int32_t>(N)), modes(B);
  std::vector<uint64_t> seeds(B);
  std::vector<float> temps(B, rq.sampling_temp);
  for (int32_t b = 0; b < B; ++b) {
    seeds[b] = rq.seed + (noisy ? (uint64_t)b : 0);
    modes[b] = rq.decode_order == InverseFoldDecodeOrder::NToC ? HKB_DECODE_N_TO_C : HKB_DECODE_RANDOM;
    std::copy(s.atom_sources, s.atom_sources + (size_t)L * 5, src.begin() + (size_t)b * L * 5);
    float* dst = coords.data() + (size_t)b * L * 15;
    if (noisy) {
      r.status = hkb_backbone_noise(L, s.coordinates, s.atom_sources, rq.backbone_noise, seeds[b], dst);
      if (r.status.code != HKB_OK) return r;
    } else {
      std::copy(s.coordinates, s.coordinates + (size_t)L * 15, dst);
    }
  }
  hkb_design_batch batch{B, lens.data(), coords.data(), src.data(), nseq.data(), seeds.data(),
                         temps.data(), modes.data(), nullptr};
  std::vector<int32_t> tokens(N * L), orders(N * L);
  std::vector<float> lp(N * L * 21), scores(N);
  hkb_design_out out{tokens.data(), lp.data(), orders.data(), scores.data()};
  r.status = hkb_mpnn_design(e_.get(), &batch, &out);
  if (r.status.code != HKB_OK) return r;
  static const char kAlphabet[] = "ACDEFGHIKLMNPQRSTVWYX";
  for (size_t i = 0; i < N; ++i) {
    InverseFoldSequenceResult q;
    q.sequence.resize(L);
    size_t cmp = 0, hit = 0;
    for (int32_t p = 0; p < L; ++p) {
      q.sequence[p] = kAlphabet[tokens[i * L + p]];
      if (s.residue_codes) {
        char nat = s.residue_codes[p];
        if (nat >= 'a' && nat <= 'z') nat = static_cast<char>(nat - 32);
        if (nat != 'X' && std::string_view("ACDEFGHIKLMNPQRSTVWY").find(nat) != std::string_view::npos) {
          ++cmp;
          hit += q.sequence[p] == nat;
        }
      }
    }
    if (cmp) q.recovery_vs_native = static_cast<double>(hit) / static_cast<double>(cmp);
    q.score = static_cast<double>(scores[i]);
    q.seed = rq.seed + i;
    q.decode_order = rq.decode_order;
    r.value.sequences.push_back(std::move(q));
  }
  if (!rq.logprobs_out.empty()) {
    r.value.logprobs = {rq.logprobs_out, N, (size_t)L, 21, std::move(lp)};
  }
  return r;
}

}  // namespace api

namespace io {

struct DesignFastaWriterOptions {
  float sampling_temp = 0.1f;
};

inline universal::Status write_design_fasta(std::string_view path, const api::InverseFoldResult& r,
                                            const DesignFastaWriterOptions& o = {}) {
  const std::string p(path);
  const size_t N = r.sequences.size();
  const int32_t L = N ? static_cast<int32_t>(r.sequences[0].sequence.size()) : 0;
  std::vector<int32_t> tok(N * L);
  std::vector<double> sc(N);
  std::vector<uint64_t> sd(N);
  static const std::string_view kAlphabet = "ACDEFGHIKLMNPQRSTVWYX";
  for (size_t i = 0; i < N; ++i) {
    for (int32_t k = 0; k < L; ++k) {
      const size_t a = kAlphabet.find(r.sequences[i].sequence[k]);
      tok[i * L + k] = a == std::string_view::npos ? 20 : static_cast<int32_t>(a);
    }
    sc[i] = r.sequences[i].score;
    sd[i] = r.sequences[i].seed;
  }
  const int32_t order = N && r.sequences[0].decode_order == api::InverseFoldDecodeOrder::NToC
                            ? HKB_DECODE_N_TO_C
                            : HKB_DECODE_RANDOM;
  return hkb_write_design_fasta(p.c_str(), static_cast<int32_t>(N), L, tok.data(), sc.data(),
                                sd.data(), o.sampling_temp, order);
}

inline universal::Status write_inverse_fold_logprobs_npz(std::string_view path,
                                                         const api::InverseFoldResult& r) {
  const std::string p(path);
  const auto& a = r.logprobs;
  if (a.values.size() != a.num_seqs * a.residue_count * a.vocab_size || a.values.empty())
    return {HKB_INVALID_ARGUMENT, "inverse-fold log-prob artifact shape is invalid"};
  return hkb_write_logprobs_npz(p.c_str(), static_cast<int32_t>(a.num_seqs),
                                static_cast<int32_t>(a.residue_count), a.values.data());
}

}  // namespace io
}  // namespace hikoboshi
