// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// C-ABI shim around the reference's own structure loader and design writers,
// compiled from the reference sources where they lie (oracle/Makefile), so the
// tests can compare the product's host IO with the reference byte for byte:
//
//   ref_load_structure   io::load_structure_from_file with default options
//                        (io/structure_loader.cpp:174-200): PDB / mmCIF parse,
//                        normalisation, atom inference, glycine virtual CB
//   ref_write_fasta      io::write_design_fasta (io/design_fasta_writer.cpp:
//                        171-199)
//   ref_write_npz        io::write_inverse_fold_logprobs_npz (:201-217)

#include <hikoboshi/api/results.hpp>
#include <hikoboshi/io/design_fasta_writer.hpp>
#include <hikoboshi/io/structure_loader.hpp>

#include <cstdint>
#include <cstring>
#include <string>

namespace {
const char* g_detail = "";
}

extern "C" {

const char* ref_io_last_detail() { return g_detail; }

// Returns the status code; on success *L is the residue count and, when the
// capacity `cap` allows, coords [L,5,3], sources [L,5] and codes [L] are filled.
int ref_load_structure(const char* path, int32_t* L, float* coords, uint8_t* sources,
                       char* codes, int32_t cap) {
  const auto r = hikoboshi::io::load_structure_from_file(path);
  g_detail = r.status.detail ? r.status.detail : "";
  if (!r.status.ok()) return static_cast<int>(r.status.code);
  const auto v = r.value.view();
  *L = static_cast<int32_t>(v.residue_count);
  if (static_cast<int64_t>(v.residue_count) > cap) return 0;
  std::memcpy(coords, v.coordinates.data, v.residue_count * 15 * sizeof(float));
  for (std::size_t i = 0; i < v.residue_count * 5; ++i)
    sources[i] = static_cast<uint8_t>(v.atom_sources.data[i]);
  std::memcpy(codes, v.residue_codes.data, v.residue_count);
  return 0;
}

// seqs: n rows of L characters.
int ref_write_fasta(const char* path, int32_t n, int32_t L, const char* seqs,
                    const double* scores, const uint64_t* seeds, float temperature,
                    int32_t n_to_c) {
  hikoboshi::api::InverseFoldResult res;
  for (int i = 0; i < n; ++i) {
    hikoboshi::api::InverseFoldSequenceResult s;
    s.sequence.assign(seqs + (size_t)i * L, (size_t)L);
    s.score = scores[i];
    s.seed = seeds[i];
    s.decode_order = n_to_c ? hikoboshi::api::InverseFoldDecodeOrder::NToC
                            : hikoboshi::api::InverseFoldDecodeOrder::Random;
    res.sequences.push_back(std::move(s));
  }
  hikoboshi::io::DesignFastaWriterOptions o{};
  o.sampling_temp = temperature;
  const auto st = hikoboshi::io::write_design_fasta(path, res, o);
  g_detail = st.detail ? st.detail : "";
  return static_cast<int>(st.code);
}

int ref_write_npz(const char* path, int32_t n, int32_t L, const float* lp) {
  hikoboshi::api::InverseFoldResult res;
  res.logprobs.num_seqs = (size_t)n;
  res.logprobs.residue_count = (size_t)L;
  res.logprobs.vocab_size = 21;
  res.logprobs.values.assign(lp, lp + (size_t)n * L * 21);
  const auto st = hikoboshi::io::write_inverse_fold_logprobs_npz(path, res);
  g_detail = st.detail ? st.detail : "";
  return static_cast<int>(st.code);
}

}  // extern "C"
