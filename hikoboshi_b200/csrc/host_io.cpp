// C ABI of the design command's host-side input and output: structure
// loading, per-sequence backbone noise, and the FASTA / NPZ writers.  The
// byte formats are the reference's (io/design_fasta_writer.cpp), since the
// output files must be drop-in identical; the code is this project's.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "hkb_mpnn.h"
#include "structure_io.hpp"

struct hkb_structure {
  hkb::io::Structure s;
};

namespace {

constexpr hkb_status kOk{HKB_OK, ""};
hkb_status bad(const char* d) { return {HKB_INVALID_ARGUMENT, d}; }
hkb_status unavailable(const char* d) { return {HKB_UNAVAILABLE, d}; }

hkb::io::LoadOptions options_of(const hkb_structure_options* o) {
  hkb::io::LoadOptions r;
  if (o) {
    r.model = o->model_index;
    r.chain = o->chain_id ? o->chain_id : "";
    r.infer_missing_atoms = o->infer_missing_atoms != 0;
    r.include_modified_residues = o->include_modified_residues != 0;
  }
  return r;
}

void put16(std::vector<uint8_t>& b, uint32_t v) {
  b.push_back(static_cast<uint8_t>(v & 0xFF));
  b.push_back(static_cast<uint8_t>((v >> 8) & 0xFF));
}
void put32(std::vector<uint8_t>& b, uint32_t v) {
  put16(b, v & 0xFFFF);
  put16(b, v >> 16);
}

// CRC-32 (IEEE 802.3, reflected polynomial 0xEDB88320), bitwise.
uint32_t crc32_of(const std::vector<uint8_t>& b) {
  uint32_t c = 0xFFFFFFFFu;
  for (const uint8_t x : b) {
    c ^= x;
    for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
  }
  return ~c;
}

}  // namespace

extern "C" {

hkb_status hkb_structure_load_text(const char* text, size_t length, int32_t format,
                                   const char* origin, const hkb_structure_options* options,
                                   hkb_structure** out) {
  if (out == nullptr) return bad("structure output pointer is null");
  *out = nullptr;
  if (text == nullptr && length > 0) return bad("structure text is null");
  const std::string_view t(text ? text : "", length);
  hkb::io::Format f = format == 1   ? hkb::io::Format::kPdb
                      : format == 2 ? hkb::io::Format::kMmcif
                                    : hkb::io::detect_format("", t);
  if (format < 0 || format > 2) return bad("structure format must be 0 (detect), 1 (PDB) or 2 (mmCIF)");
  if (f == hkb::io::Format::kUnknown)
    return bad("unrecognized structure file format; extension and content cues did not match "
               "PDB or mmCIF");
  auto* h = new hkb_structure;
  const hkb_status st = hkb::io::load_text(t, f, origin ? origin : "", options_of(options), &h->s);
  if (st.code != HKB_OK) {
    delete h;
    return st;
  }
  *out = h;
  return kOk;
}

hkb_status hkb_structure_load_file(const char* path, const hkb_structure_options* options,
                                   hkb_structure** out) {
  if (out == nullptr) return bad("structure output pointer is null");
  *out = nullptr;
  if (path == nullptr || path[0] == '\0') return bad("structure path is required");
  auto* h = new hkb_structure;
  const hkb_status st = hkb::io::load_file(path, options_of(options), &h->s);
  if (st.code != HKB_OK) {
    delete h;
    return st;
  }
  *out = h;
  return kOk;
}

int32_t hkb_structure_residue_count(const hkb_structure* s) { return s ? s->s.L : 0; }

hkb_status hkb_structure_copy(const hkb_structure* s, float* coords, uint8_t* atom_sources,
                              char* residue_codes) {
  if (s == nullptr) return bad("structure is null");
  const size_t L = static_cast<size_t>(s->s.L);
  if (coords) std::memcpy(coords, s->s.coords.data(), L * 15 * sizeof(float));
  if (atom_sources) std::memcpy(atom_sources, s->s.sources.data(), L * 5);
  if (residue_codes) std::memcpy(residue_codes, s->s.codes.data(), L);
  return kOk;
}

void hkb_structure_destroy(hkb_structure* s) { delete s; }

hkb_status hkb_backbone_noise(int32_t residue_count, const float* coords,
                              const uint8_t* atom_sources, float sigma, uint64_t seed,
                              float* out) {
  if (residue_count <= 0 || coords == nullptr || atom_sources == nullptr || out == nullptr)
    return bad("inverse-fold structure must provide canonical backbone atoms");
  if (!std::isfinite(sigma) || sigma < 0.0f)
    return bad("inverse-fold backbone_noise must be finite and >= 0");
  const size_t n = static_cast<size_t>(residue_count) * 5;
  if (out != coords) std::memcpy(out, coords, n * 3 * sizeof(float));
  if (!(sigma > 0.0f)) return kOk;
  std::mt19937_64 engine(seed ^ 0x4D504E4E76343875ull);
  std::normal_distribution<float> gauss(0.0f, sigma);
  for (size_t a = 0; a < n; ++a) {
    if (atom_sources[a] == hkb::io::kSrcMissing) continue;
    for (int x = 0; x < 3; ++x) out[a * 3 + x] += gauss(engine);
  }
  return kOk;
}

hkb_status hkb_write_design_fasta(const char* path, int32_t num_seqs, int32_t residue_count,
                                  const int32_t* tokens, const double* scores,
                                  const uint64_t* seeds, float sampling_temp,
                                  int32_t decode_order) {
  if (path == nullptr || path[0] == '\0') return bad("design FASTA output path is required");
  if (num_seqs < 0 || residue_count < 0 || (num_seqs > 0 && (!tokens || !scores || !seeds)))
    return bad("design FASTA input is invalid");
  static const char kAlphabet[] = "ACDEFGHIKLMNPQRSTVWYX";
  std::ofstream f(path);
  if (!f) return unavailable("design FASTA output is not writable");
  std::string seq(static_cast<size_t>(residue_count), 'X');
  for (int32_t i = 0; i < num_seqs; ++i) {
    for (int32_t p = 0; p < residue_count; ++p) {
      const int32_t t = tokens[(size_t)i * residue_count + p];
      seq[p] = (t >= 0 && t < 21) ? kAlphabet[t] : 'X';
    }
    // ostream formatting as the reference writes it: 7 significant digits
    // (setprecision persists for T), seed as an unsigned integer
    f << ">design_" << (i + 1) << " score=" << std::setprecision(7) << scores[i]
      << " seed=" << seeds[i] << " T=" << sampling_temp
      << " decode_order=" << (decode_order == HKB_DECODE_N_TO_C ? "n_to_c" : "random") << "\n";
    for (int32_t o = 0; o < residue_count; o += 80) {
      f.write(seq.data() + o, std::min<int32_t>(80, residue_count - o));
      f << "\n";
    }
  }
  if (!f) return unavailable("design FASTA output could not be written");
  return kOk;
}

hkb_status hkb_write_logprobs_npz(const char* path, int32_t num_seqs, int32_t residue_count,
                                  const float* log_probs) {
  if (path == nullptr || path[0] == '\0')
    return bad("inverse-fold log-prob output path is required");
  if (num_seqs <= 0 || residue_count <= 0 || log_probs == nullptr)
    return bad("inverse-fold log-prob artifact shape is invalid");
  // .npy v1.0: magic, version, u16 header length, dict padded with blanks to
  // a 16-byte boundary and ended by a newline, little-endian f4 data
  std::vector<uint8_t> npy = {0x93, 'N', 'U', 'M', 'P', 'Y', 1, 0};
  std::ostringstream h;
  h << "{'descr': '<f4', 'fortran_order': False, 'shape': (" << num_seqs << ", "
    << residue_count << ", 21), }";
  std::string hdr = h.str();
  hdr.append((16 - (10 + hdr.size() + 1) % 16) % 16, ' ');
  hdr.push_back('\n');
  put16(npy, static_cast<uint32_t>(hdr.size()));
  npy.insert(npy.end(), hdr.begin(), hdr.end());
  const size_t n = (size_t)num_seqs * residue_count * 21;
  for (size_t i = 0; i < n; ++i) {
    uint32_t bits;
    std::memcpy(&bits, &log_probs[i], 4);
    put32(npy, bits);
  }
  if (npy.size() > 0xFFFFFFFFull) return bad("inverse-fold log-prob artifact is too large for ZIP32");
  // ZIP32, one stored member: local header, data, central directory, end record
  const std::string name = "log_probs.npy";
  const uint32_t size = static_cast<uint32_t>(npy.size()), crc = crc32_of(npy);
  std::vector<uint8_t> z;
  auto member_fields = [&](bool central) {
    put16(z, 20);                      // version needed (central: made by, then needed)
    if (central) put16(z, 20);
    for (int k = 0; k < 4; ++k) put16(z, 0);   // flags, method (stored), time, date
    put32(z, crc);
    put32(z, size);
    put32(z, size);
    put16(z, static_cast<uint32_t>(name.size()));
    put16(z, 0);                       // extra length
  };
  put32(z, 0x04034B50u);
  member_fields(false);
  z.insert(z.end(), name.begin(), name.end());
  z.insert(z.end(), npy.begin(), npy.end());
  if (z.size() > 0xFFFFFFFFull) return bad("inverse-fold log-prob artifact is too large for ZIP32");
  const uint32_t cd_off = static_cast<uint32_t>(z.size());
  put32(z, 0x02014B50u);
  member_fields(true);
  put16(z, 0);   // comment length
  put16(z, 0);   // disk number
  put16(z, 0);   // internal attributes
  put32(z, 0);   // external attributes
  put32(z, 0);   // local header offset
  z.insert(z.end(), name.begin(), name.end());
  const uint32_t cd_size = static_cast<uint32_t>(z.size()) - cd_off;
  put32(z, 0x06054B50u);
  put16(z, 0);
  put16(z, 0);
  put16(z, 1);
  put16(z, 1);
  put32(z, cd_size);
  put32(z, cd_off);
  put16(z, 0);
  std::ofstream f(path, std::ios::binary);
  if (!f) return unavailable("inverse-fold log-prob artifact is not writable");
  f.write(reinterpret_cast<const char*>(z.data()), static_cast<std::streamsize>(z.size()));
  if (!f) return unavailable("inverse-fold log-prob artifact could not be written");
  return kOk;
}

}  // extern "C"
