// Host-side structure input for the design path: PDB / mmCIF text -> the
// canonical [L,5,3] backbone (N, CA, C, O, CB) plus per-atom sources, the way
// the reference's loader produces it (io/structure_loader.cpp:174-284,
// io/pdb_parser.cpp, io/mmcif_parser.cpp, io/structure_normalize.cpp,
// io/atom_inference.cpp, io/virtual_cb.cpp, io/residue_table.cpp).
#pragma once

#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

#include "hkb_mpnn.h"

namespace hkb::io {

// Atom provenance, the reference's universal::AtomSource values.
enum : uint8_t { kSrcMissing = 0, kSrcObserved = 1, kSrcInferred = 2, kSrcVirtual = 3 };

// One ATOM / HETATM row as read, before model / chain / altloc selection.
struct AtomRow {
  int64_t record = 0;        // index among the file's atom rows
  bool hetatm = false;
  int32_t model = 1;
  std::string model_id = "1";
  std::string atom;          // atom name, trimmed
  std::string residue;       // residue name, trimmed
  std::string chain;
  char altloc = ' ';
  int32_t resnum = 0;
  char icode = ' ';
  float x = 0.0f, y = 0.0f, z = 0.0f;
};

struct LoadOptions {
  int32_t model = 0;                 // 0: the reference default (model 1)
  std::string chain;                 // empty: "A" if present, else the first polymer chain
  bool infer_missing_atoms = true;
  bool include_modified_residues = true;
};

// A normalised single chain.
struct Structure {
  int32_t L = 0;
  std::vector<float> coords;         // [L,5,3]
  std::vector<uint8_t> sources;      // [L,5]
  std::string codes;                 // [L] one-letter codes ('X' unknown)
  std::string chain_id, model_id;
  std::string origin;                // file name without directories
};

enum class Format { kUnknown, kPdb, kMmcif };

Format detect_format(std::string_view path, std::string_view text);
hkb_status parse_pdb(std::string_view text, std::vector<AtomRow>* rows);
hkb_status parse_mmcif(std::string_view text, std::vector<AtomRow>* rows);
hkb_status normalize(const std::vector<AtomRow>& rows, const LoadOptions& opt, Structure* out);
void infer_missing_atoms(Structure* s);
hkb_status load_text(std::string_view text, Format fmt, std::string_view origin,
                     const LoadOptions& opt, Structure* out);
hkb_status load_file(const std::string& path, const LoadOptions& opt, Structure* out);

// Glycine virtual CB from N, CA, C (io/virtual_cb.cpp:16-38).
void virtual_cb(const float n[3], const float ca[3], const float c[3], float out[3]);

}  // namespace hkb::io
