// Structure input: PDB / mmCIF -> canonical backbone.  Behaviour follows the
// reference loader (file:line cited per function); the code is this project's.
#include "structure_io.hpp"

#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>
#include <unordered_map>
#include <unordered_set>

namespace hkb::io {
namespace {

constexpr hkb_status kOk{HKB_OK, ""};
hkb_status bad(const char* d) { return {HKB_INVALID_ARGUMENT, d}; }

bool begins(std::string_view s, std::string_view p) {
  return s.size() >= p.size() && s.compare(0, p.size(), p) == 0;
}

bool is_ws(char c) { return std::isspace(static_cast<unsigned char>(c)) != 0; }

// PDB column fields drop blanks, tabs and a trailing CR (pdb_parser.cpp:20-33).
std::string_view trim_pdb(std::string_view s) {
  size_t b = 0, e = s.size();
  while (b < e && (s[b] == ' ' || s[b] == '\t')) ++b;
  while (e > b && (s[e - 1] == ' ' || s[e - 1] == '\t' || s[e - 1] == '\r')) --e;
  return s.substr(b, e - b);
}

// mmCIF tokens drop any white space (mmcif_parser.cpp:25-36).
std::string_view trim_ws(std::string_view s) {
  size_t b = 0, e = s.size();
  while (b < e && is_ws(s[b])) ++b;
  while (e > b && is_ws(s[e - 1])) --e;
  return s.substr(b, e - b);
}

std::string_view field(std::string_view line, size_t pos, size_t n) {
  if (pos >= line.size()) return {};
  return line.substr(pos, std::min(n, line.size() - pos));
}

// Integer / real fields: optional leading '+', the whole (trimmed) field must
// parse; reals must be finite and are read as double, then narrowed.
bool to_int(std::string_view s, int32_t* out) {
  if (!s.empty() && s.front() == '+') s.remove_prefix(1);
  if (s.empty()) return false;
  int64_t v = 0;
  const auto r = std::from_chars(s.data(), s.data() + s.size(), v);
  if (r.ec != std::errc{} || r.ptr != s.data() + s.size()) return false;
  *out = static_cast<int32_t>(v);
  return true;
}

bool to_real(std::string_view s, float* out) {
  if (!s.empty() && s.front() == '+') s.remove_prefix(1);
  if (s.empty()) return false;
  double v = 0.0;
  const auto r = std::from_chars(s.data(), s.data() + s.size(), v);
  if (r.ec != std::errc{} || r.ptr != s.data() + s.size() || !std::isfinite(v)) return false;
  *out = static_cast<float>(v);
  return true;
}

bool ends_with_nocase(std::string_view s, std::string_view suf) {
  if (s.size() < suf.size()) return false;
  for (size_t i = 0; i < suf.size(); ++i) {
    char a = s[s.size() - suf.size() + i];
    if (a >= 'A' && a <= 'Z') a = static_cast<char>(a + 32);
    if (a != suf[i]) return false;
  }
  return true;
}

// Calls f(line) for each '\n'-separated line (a last line without newline
// included); f returns false to stop.
template <typename F>
void for_lines(std::string_view text, F f) {
  size_t pos = 0;
  while (pos <= text.size()) {
    const size_t e = text.find('\n', pos);
    const std::string_view line = text.substr(pos, e == std::string_view::npos ? text.size() - pos
                                                                                : e - pos);
    if (!f(line)) return;
    if (e == std::string_view::npos) return;
    pos = e + 1;
  }
}

}  // namespace

// Extension first, then content cues (structure_loader.cpp:101-172).
Format detect_format(std::string_view path, std::string_view text) {
  if (ends_with_nocase(path, ".cif") || ends_with_nocase(path, ".mmcif")) return Format::kMmcif;
  if (ends_with_nocase(path, ".pdb") || ends_with_nocase(path, ".ent")) return Format::kPdb;
  if (begins(text, "data_") || text.find("_atom_site.") != std::string_view::npos)
    return Format::kMmcif;
  bool pdb = false;
  for_lines(text, [&](std::string_view line) {
    if (line.size() >= 6 && (begins(line, "ATOM  ") || begins(line, "HETATM") ||
                             begins(line, "MODEL "))) {
      pdb = true;
      return false;
    }
    return true;
  });
  return pdb ? Format::kPdb : Format::kUnknown;
}

// Fixed-column ATOM / HETATM rows with MODEL / ENDMDL bracketing
// (pdb_parser.cpp:101-196).  Rows outside a MODEL block belong to model 1.
hkb_status parse_pdb(std::string_view text, std::vector<AtomRow>* rows) {
  rows->clear();
  int32_t model = 1;
  bool in_model = false;
  hkb_status st = kOk;
  for_lines(text, [&](std::string_view line) {
    if (begins(line, "MODEL ")) {
      int32_t m = 0;
      if (!to_int(trim_pdb(field(line, 10, 4)), &m)) {
        st = bad("PDB MODEL record missing or unparseable serial");
        return false;
      }
      model = m;
      in_model = true;
    } else if (begins(line, "ENDMDL")) {
      in_model = false;
    } else if (begins(line, "ATOM  ") || begins(line, "HETATM")) {
      if (line.size() < 54) {
        st = bad("PDB ATOM/HETATM record shorter than the 54-column coordinate block");
        return false;
      }
      AtomRow a;
      a.record = static_cast<int64_t>(rows->size());
      a.hetatm = begins(line, "HETATM");
      a.model = in_model ? model : 1;
      a.model_id = std::to_string(a.model);
      int32_t serial = 0;
      if (!to_int(trim_pdb(field(line, 6, 5)), &serial)) {
        st = bad("PDB ATOM/HETATM record has invalid serial column");
        return false;
      }
      a.atom = std::string(trim_pdb(field(line, 12, 4)));
      a.altloc = line[16];
      a.residue = std::string(trim_pdb(field(line, 17, 3)));
      a.chain = std::string(trim_pdb(field(line, 21, 1)));
      if (!to_int(trim_pdb(field(line, 22, 4)), &a.resnum)) {
        st = bad("PDB ATOM/HETATM record has invalid residue number");
        return false;
      }
      const std::string_view ic = field(line, 26, 1);
      a.icode = ic.empty() ? ' ' : ic.front();
      if (!to_real(trim_pdb(field(line, 30, 8)), &a.x) ||
          !to_real(trim_pdb(field(line, 38, 8)), &a.y) ||
          !to_real(trim_pdb(field(line, 46, 8)), &a.z)) {
        st = bad("PDB ATOM/HETATM record has invalid coordinate field; refusing to silently "
                 "zero-fill");
        return false;
      }
      rows->push_back(std::move(a));
    }
    return true;
  });
  return st;
}

namespace {

// Whitespace-separated tokens; a token that starts with ' or " runs to the
// matching quote (mmcif_parser.cpp:65-98).  No ;-delimited text fields.
void cif_tokens(std::string_view line, std::vector<std::string>* out) {
  size_t i = 0;
  while (i < line.size()) {
    while (i < line.size() && is_ws(line[i])) ++i;
    if (i >= line.size()) break;
    if (line[i] == '"' || line[i] == '\'') {
      const char q = line[i++];
      const size_t b = i;
      while (i < line.size() && line[i] != q) ++i;
      out->emplace_back(line.substr(b, i - b));
      if (i < line.size()) ++i;
    } else {
      const size_t b = i;
      while (i < line.size() && !is_ws(line[i])) ++i;
      out->emplace_back(line.substr(b, i - b));
    }
  }
}

// Line cursor over the text: current line and the offset after it.
struct Cursor {
  std::string_view text;
  size_t pos = 0;
  bool done() const { return pos > text.size(); }
  std::string_view line(size_t* next) const {
    const size_t e = text.find('\n', pos);
    *next = e == std::string_view::npos ? text.size() + 1 : e + 1;
    return text.substr(pos, e == std::string_view::npos ? text.size() - pos : e - pos);
  }
};

}  // namespace

// _atom_site loop rows of every data block (mmcif_parser.cpp:101-343).  Name,
// residue, chain and number prefer the label_ / auth_ columns the reference
// prefers; rows may wrap over several lines.
hkb_status parse_mmcif(std::string_view text, std::vector<AtomRow>* rows) {
  rows->clear();
  bool found = false;
  Cursor c{text, 0};
  constexpr size_t kNone = static_cast<size_t>(-1);
  while (!c.done()) {
    size_t next = 0;
    const std::string_view line = trim_ws(c.line(&next));
    if (!begins(line, "loop_")) {
      c.pos = next;
      continue;
    }
    // column declarations
    std::vector<std::string> cols;
    bool atom_site = false;
    Cursor s{text, next};
    while (!s.done()) {
      size_t n2 = 0;
      const std::string_view t = trim_ws(s.line(&n2));
      if (begins(t, "_atom_site.")) {
        atom_site = true;
        cols.emplace_back(t.substr(11));
      } else if (begins(t, "_")) {
        cols.clear();
        break;
      } else if (!t.empty()) {
        break;   // first data row
      }
      s.pos = n2;
    }
    if (!atom_site || cols.empty()) {
      c.pos = next;
      continue;
    }
    found = true;
    std::unordered_map<std::string, size_t> at;
    for (size_t i = 0; i < cols.size(); ++i) at[cols[i]] = i;
    auto col = [&](const char* n) {
      const auto it = at.find(n);
      return it == at.end() ? kNone : it->second;
    };
    auto either = [&](const char* a, const char* b) { return col(a) != kNone ? col(a) : col(b); };
    const size_t k_group = col("group_PDB"), k_alt = col("label_alt_id");
    const size_t k_name = either("label_atom_id", "auth_atom_id");
    const size_t k_res = either("auth_comp_id", "label_comp_id");
    const size_t k_chain = either("auth_asym_id", "label_asym_id");
    const size_t k_num = either("auth_seq_id", "label_seq_id");
    const size_t k_ins = col("pdbx_PDB_ins_code"), k_model = col("pdbx_PDB_model_num");
    const size_t kx = col("Cartn_x"), ky = col("Cartn_y"), kz = col("Cartn_z");
    if (k_name == kNone) return bad("mmCIF _atom_site loop missing required atom-name column");
    if (kx == kNone || ky == kNone || kz == kNone)
      return bad("mmCIF _atom_site loop missing required Cartesian coordinate columns");
    c.pos = s.pos;
    while (!c.done()) {
      size_t n3 = 0;
      const std::string_view r = trim_ws(c.line(&n3));
      if (r.empty()) {
        c.pos = n3;
        continue;
      }
      if (begins(r, "loop_") || begins(r, "data_") || begins(r, "_") || begins(r, "#")) break;
      std::vector<std::string> tok;
      cif_tokens(r, &tok);
      while (tok.size() < cols.size() && n3 < text.size()) {   // wrapped row
        Cursor w{text, n3};
        cif_tokens(trim_ws(w.line(&n3)), &tok);
      }
      if (tok.size() < cols.size()) return bad("mmCIF _atom_site row column count mismatch");
      AtomRow a;
      a.record = static_cast<int64_t>(rows->size());
      a.hetatm = (k_group == kNone ? tok[0] : tok[k_group]) == "HETATM";
      a.atom = tok[k_name];
      if (k_alt != kNone) {
        const std::string& v = tok[k_alt];
        a.altloc = (v == "." || v == "?") ? ' ' : v.front();
      }
      if (k_res != kNone) a.residue = tok[k_res];
      if (k_chain != kNone) {
        const std::string& v = tok[k_chain];
        a.chain = (v == "." || v == "?") ? std::string() : v;
      }
      if (k_num != kNone && !to_int(trim_ws(tok[k_num]), &a.resnum))
        return bad("mmCIF _atom_site row has unparseable residue number");
      if (k_ins != kNone) {
        const std::string& v = tok[k_ins];
        a.icode = (v == "?" || v == "." || v.empty()) ? ' ' : v.front();
      }
      auto coord = [&](size_t k, float* o) {
        const std::string_view v = trim_ws(tok[k]);
        return !(v == "?" || v == ".") && to_real(v, o);
      };
      if (!coord(kx, &a.x) || !coord(ky, &a.y) || !coord(kz, &a.z))
        return bad("mmCIF _atom_site row has unparseable coordinate; refusing to silently "
                   "zero-fill");
      int32_t m = 1;
      if (k_model != kNone && to_int(trim_ws(tok[k_model]), &m)) {
        a.model = m;
        a.model_id = tok[k_model];
      }
      rows->push_back(std::move(a));
      c.pos = n3;
    }
  }
  if (!found) return bad("mmCIF input does not contain an _atom_site loop");
  return kOk;
}

namespace {

// The 20 canonical amino acids and the modified residues read as their parent
// (residue_table.cpp:15-40), matched case-insensitively on the trimmed name.
char residue_letter(std::string_view name, bool* modified) {
  static const char* kCanon[20] = {"ALA", "ARG", "ASN", "ASP", "CYS", "GLN", "GLU",
                                   "GLY", "HIS", "ILE", "LEU", "LYS", "MET", "PHE",
                                   "PRO", "SER", "THR", "TRP", "TYR", "VAL"};
  static const char kCanonLetter[] = "ARNDCQEGHILKMFPSTWYV";
  static const char* kMod[7] = {"MSE", "SEC", "PYL", "SEP", "TPO", "PTR", "HYP"};
  static const char kModLetter[] = "MCKSTYP";
  name = trim_pdb(name);
  char up[4] = {0, 0, 0, 0};
  const bool three = name.size() == 3;
  for (size_t i = 0; three && i < 3; ++i)
    up[i] = (name[i] >= 'a' && name[i] <= 'z') ? static_cast<char>(name[i] - 32) : name[i];
  *modified = false;
  if (!three) return 'X';
  for (int i = 0; i < 20; ++i)
    if (std::memcmp(up, kCanon[i], 3) == 0) return kCanonLetter[i];
  for (int i = 0; i < 7; ++i)
    if (std::memcmp(up, kMod[i], 3) == 0) {
      *modified = true;
      return kModLetter[i];
    }
  return 'X';
}

int slot_of(const std::string& atom) {
  if (atom == "N") return 0;
  if (atom == "CA") return 1;
  if (atom == "C") return 2;
  if (atom == "O") return 3;
  if (atom == "CB") return 4;
  return -1;
}

// Backbone atoms of ATOM rows, and of HETATM rows of whitelisted modified
// residues (structure_normalize.cpp:78-91).
bool polymer_atom(const AtomRow& a, const LoadOptions& o) {
  if (slot_of(a.atom) < 0) return false;
  if (!a.hetatm) return true;
  bool mod = false;
  const char l = residue_letter(a.residue, &mod);
  return o.include_modified_residues && mod && l != 'X';
}

int altloc_rank(char c) {
  if (c == ' ' || c == '\0') return 0;
  if (c == 'A' || c == 'a') return 1;
  return 2;
}

}  // namespace

// Model, chain, altloc and residue grouping (structure_normalize.cpp:93-362):
// model 1 unless asked; chain "A" if present among polymer rows, else the
// first; residues keyed by (chain, number, insertion code) in first-seen
// order; per atom, a blank altloc wins for good, then 'A', then the first seen.
hkb_status normalize(const std::vector<AtomRow>& rows, const LoadOptions& o, Structure* out) {
  const int32_t model = o.model != 0 ? o.model : 1;
  const AtomRow* first = nullptr;
  for (const AtomRow& a : rows)
    if (a.model == model) {
      first = &a;
      break;
    }
  if (!first) return bad("selected model index not present in input");
  std::vector<std::string> chains;
  std::unordered_set<std::string> seen;
  for (const AtomRow& a : rows)
    if (a.model == model && polymer_atom(a, o) && seen.insert(a.chain).second)
      chains.push_back(a.chain);
  std::string chain;
  if (!o.chain.empty()) {
    if (!seen.count(o.chain)) return bad("requested chain id not present in selected model");
    chain = o.chain;
  } else if (seen.count("A")) {
    chain = "A";
  } else if (!chains.empty()) {
    chain = chains.front();
  } else {
    return bad("selected model has no polymer chains");
  }
  struct Res {
    char code;
    float xyz[5][3] = {};
    uint8_t src[5] = {0, 0, 0, 0, 0};
    char alt[5] = {' ', ' ', ' ', ' ', ' '};
    bool blank[5] = {false, false, false, false, false};
  };
  std::vector<Res> res;
  std::map<std::tuple<int32_t, char>, size_t> index;   // chain is fixed
  for (const AtomRow& a : rows) {
    if (a.model != model || a.chain != chain || !polymer_atom(a, o)) continue;
    const int k = slot_of(a.atom);
    auto it = index.find({a.resnum, a.icode});
    if (it == index.end()) {
      Res r;
      bool mod = false;
      r.code = residue_letter(a.residue, &mod);
      res.push_back(r);
      it = index.emplace(std::make_tuple(a.resnum, a.icode), res.size() - 1).first;
    }
    Res& r = res[it->second];
    if (r.src[k] == kSrcObserved) {
      if (r.blank[k]) continue;
      const bool take = (a.altloc == ' ' || a.altloc == '\0') ||
                        altloc_rank(a.altloc) < altloc_rank(r.alt[k]);
      if (!take) continue;
    }
    r.xyz[k][0] = a.x;
    r.xyz[k][1] = a.y;
    r.xyz[k][2] = a.z;
    r.src[k] = kSrcObserved;
    if (a.altloc == ' ' || a.altloc == '\0') r.blank[k] = true;
    r.alt[k] = a.altloc;
  }
  if (res.empty()) return bad("selected chain has no accepted amino-acid residues");
  out->L = static_cast<int32_t>(res.size());
  out->coords.assign(res.size() * 15, 0.0f);
  out->sources.assign(res.size() * 5, kSrcMissing);
  out->codes.assign(res.size(), 'X');
  for (size_t i = 0; i < res.size(); ++i) {
    out->codes[i] = res[i].code;
    for (int k = 0; k < 5; ++k) {
      out->sources[i * 5 + k] = res[i].src[k];
      if (res[i].src[k] == kSrcObserved)
        for (int x = 0; x < 3; ++x) out->coords[i * 15 + k * 3 + x] = res[i].xyz[k][x];
    }
  }
  out->chain_id = chain;
  out->model_id = first->model_id;
  return kOk;
}

// Glycine virtual CB: CA + a (b x c) + b' b + c' c with b = CA - N,
// c = C - CA and the ProteinMPNN coefficients (virtual_cb.cpp:16-38).
void virtual_cb(const float n[3], const float ca[3], const float c[3], float out[3]) {
  const float b[3] = {ca[0] - n[0], ca[1] - n[1], ca[2] - n[2]};
  const float cv[3] = {c[0] - ca[0], c[1] - ca[1], c[2] - ca[2]};
  const float a[3] = {b[1] * cv[2] - b[2] * cv[1], b[2] * cv[0] - b[0] * cv[2],
                      b[0] * cv[1] - b[1] * cv[0]};
  for (int x = 0; x < 3; ++x)
    out[x] = ca[x] + -0.58273431f * a[x] + 0.56802827f * b[x] + -0.54067466f * cv[x];
}

namespace {

// Ideal residue in a local frame (residue_table.cpp:61-115): CA at the
// origin, N on -x, C in the xy plane at the N-CA-C angle, O in the plane at
// the CA-C-O angle, CB by the virtual-CB rule.  Float arithmetic in the
// reference's order, so the template is the same to the last bit.
struct Template {
  float xyz[5][3];
};

const Template& ideal_residue() {
  static const Template t = [] {
    Template r{};
    const float d_nca = 1.458f, d_cac = 1.525f, d_co = 1.231f;
    const float a_ncac = 1.9416f, a_caco = 2.1031f;
    const float ca[3] = {0.0f, 0.0f, 0.0f};
    const float n[3] = {-d_nca, 0.0f, 0.0f};
    const float cc[3] = {d_cac * std::cos(a_ncac - 1.5707963267948966f),
                         d_cac * std::sin(a_ncac - 1.5707963267948966f), 0.0f};
    const float dv[3] = {cc[0] - ca[0], cc[1] - ca[1], cc[2] - ca[2]};
    const float len = std::sqrt(dv[0] * dv[0] + dv[1] * dv[1] + dv[2] * dv[2]);
    const float u[3] = {dv[0] / len, dv[1] / len, dv[2] / len};
    const float w[3] = {-u[1], u[0], 0.0f};
    const float co = std::cos(3.14159265358979f - a_caco);
    const float so = std::sin(3.14159265358979f - a_caco);
    const float dir[3] = {co * u[0] + so * w[0], co * u[1] + so * w[1], co * u[2] + so * w[2]};
    const float o[3] = {cc[0] + d_co * dir[0], cc[1] + d_co * dir[1], cc[2] + d_co * dir[2]};
    float cb[3];
    virtual_cb(n, ca, cc, cb);
    const float* p[5] = {n, ca, cc, o, cb};
    for (int k = 0; k < 5; ++k)
      for (int x = 0; x < 3; ++x) r.xyz[k][x] = p[k][x];
    return r;
  }();
  return t;
}

using M3 = double[3][3];

// Symmetric 3x3 eigen-decomposition by cyclic Jacobi rotations (at most 64
// sweeps, stop when the off-diagonal sum is below 1e-12); columns of v are
// the eigenvectors.
void jacobi3(M3 a, M3 v, double d[3]) {
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) v[i][j] = i == j ? 1.0 : 0.0;
  for (int sweep = 0; sweep < 64; ++sweep) {
    const double off = std::fabs(a[0][1]) + std::fabs(a[0][2]) + std::fabs(a[1][2]);
    if (off < 1e-12) break;
    for (int p = 0; p < 3; ++p)
      for (int q = p + 1; q < 3; ++q) {
        const double app = a[p][p], aqq = a[q][q], apq = a[p][q];
        if (std::fabs(apq) < 1e-15) continue;
        const double th = (aqq - app) / (2.0 * apq);
        const double t = th >= 0.0 ? 1.0 / (th + std::sqrt(1.0 + th * th))
                                   : 1.0 / (th - std::sqrt(1.0 + th * th));
        const double cs = 1.0 / std::sqrt(1.0 + t * t), sn = t * cs;
        a[p][p] = app - t * apq;
        a[q][q] = aqq + t * apq;
        a[p][q] = a[q][p] = 0.0;
        for (int r = 0; r < 3; ++r) {
          if (r == p || r == q) continue;
          const double arp = a[r][p], arq = a[r][q];
          a[r][p] = a[p][r] = cs * arp - sn * arq;
          a[r][q] = a[q][r] = sn * arp + cs * arq;
        }
        for (int r = 0; r < 3; ++r) {
          const double vp = v[r][p], vq = v[r][q];
          v[r][p] = cs * vp - sn * vq;
          v[r][q] = sn * vp + cs * vq;
        }
      }
  }
  for (int i = 0; i < 3; ++i) d[i] = a[i][i];
}

void mul3(const M3 a, const M3 b, M3 o) {
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      double s = 0.0;
      for (int k = 0; k < 3; ++k) s += a[i][k] * b[k][j];
      o[i][j] = s;
    }
}

// Least-squares rigid fit q ~ R p + t of n >= 3 point pairs (Kabsch): R from
// the eigenvectors of H^T H, H = sum (p - p0)(q - q0)^T, with a reflection
// fix; false when the anchors are (nearly) collinear.  rmsd over the pairs.
bool rigid_fit(const double (*p)[3], const double (*q)[3], int n, M3 R, double t[3],
               double* rmsd) {
  double cp[3] = {0, 0, 0}, cq[3] = {0, 0, 0};
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < 3; ++j) {
      cp[j] += p[i][j];
      cq[j] += q[i][j];
    }
  for (int j = 0; j < 3; ++j) {
    cp[j] /= n;
    cq[j] /= n;
  }
  M3 H = {{0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  for (int i = 0; i < n; ++i) {
    const double a[3] = {p[i][0] - cp[0], p[i][1] - cp[1], p[i][2] - cp[2]};
    const double b[3] = {q[i][0] - cq[0], q[i][1] - cq[1], q[i][2] - cq[2]};
    for (int x = 0; x < 3; ++x)
      for (int y = 0; y < 3; ++y) H[x][y] += a[x] * b[y];
  }
  M3 Ht, HtH, E;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) Ht[i][j] = H[j][i];
  mul3(Ht, H, HtH);
  double ev[3];
  jacobi3(HtH, E, ev);
  int ord[3] = {0, 1, 2};   // eigenvalues descending
  for (int i = 0; i < 3; ++i)
    for (int j = i + 1; j < 3; ++j)
      if (ev[ord[j]] > ev[ord[i]]) std::swap(ord[i], ord[j]);
  double lam[3];
  M3 V;
  for (int i = 0; i < 3; ++i) {
    lam[i] = ev[ord[i]];
    for (int j = 0; j < 3; ++j) V[j][i] = E[j][ord[i]];
  }
  if (lam[0] <= 1e-12 || lam[1] <= 1e-12) return false;
  double sig[3];
  for (int i = 0; i < 3; ++i) sig[i] = std::sqrt(std::max(0.0, lam[i]));
  M3 U = {{0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
  for (int j = 0; j < 2; ++j)
    for (int i = 0; i < 3; ++i) {
      double s = 0.0;
      for (int k = 0; k < 3; ++k) s += H[i][k] * V[k][j];
      U[i][j] = sig[j] > 1e-12 ? s / sig[j] : 0.0;
    }
  U[0][2] = U[1][0] * U[2][1] - U[2][0] * U[1][1];
  U[1][2] = U[2][0] * U[0][1] - U[0][0] * U[2][1];
  U[2][2] = U[0][0] * U[1][1] - U[1][0] * U[0][1];
  M3 Ut, VUt;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) Ut[i][j] = U[j][i];
  mul3(V, Ut, VUt);
  const double det = VUt[0][0] * (VUt[1][1] * VUt[2][2] - VUt[1][2] * VUt[2][1]) -
                     VUt[0][1] * (VUt[1][0] * VUt[2][2] - VUt[1][2] * VUt[2][0]) +
                     VUt[0][2] * (VUt[1][0] * VUt[2][1] - VUt[1][1] * VUt[2][0]);
  if (det < 0.0)
    for (int i = 0; i < 3; ++i) V[i][2] = -V[i][2];
  mul3(V, Ut, R);
  for (int i = 0; i < 3; ++i) t[i] = cq[i] - (R[i][0] * cp[0] + R[i][1] * cp[1] + R[i][2] * cp[2]);
  double err = 0.0;
  for (int i = 0; i < n; ++i)
    for (int a = 0; a < 3; ++a) {
      const double m = R[a][0] * p[i][0] + R[a][1] * p[i][1] + R[a][2] * p[i][2] + t[a];
      err += (m - q[i][a]) * (m - q[i][a]);
    }
  *rmsd = std::sqrt(err / static_cast<double>(n));
  return true;
}

}  // namespace

// Fills missing backbone atoms (atom_inference.cpp:36-110,
// atom_inference_kabsch.cpp:224-305): glycine gets the virtual CB (marked
// Virtual only when N, CA and C were observed; the coordinates are written
// either way), every other residue with >= 3 observed atoms a rigid fit of
// the ideal residue, applied only when its RMSD is <= 0.5 A.
void infer_missing_atoms(Structure* s) {
  const Template& tp = ideal_residue();
  for (int32_t i = 0; i < s->L; ++i) {
    float* x = s->coords.data() + (size_t)i * 15;
    uint8_t* src = s->sources.data() + (size_t)i * 5;
    if (s->codes[i] == 'G') {
      if (src[4] != kSrcMissing) continue;
      float cb[3];
      virtual_cb(x, x + 3, x + 6, cb);
      for (int k = 0; k < 3; ++k) x[12 + k] = cb[k];
      const bool anchored =
          src[0] == kSrcObserved && src[1] == kSrcObserved && src[2] == kSrcObserved;
      src[4] = anchored ? kSrcVirtual : kSrcMissing;
      continue;
    }
    double p[5][3], q[5][3];
    int n = 0, miss[5], nm = 0;
    for (int k = 0; k < 5; ++k) {
      if (src[k] == kSrcObserved) {
        for (int a = 0; a < 3; ++a) {
          p[n][a] = tp.xyz[k][a];
          q[n][a] = x[k * 3 + a];
        }
        ++n;
      } else if (src[k] == kSrcMissing) {
        miss[nm++] = k;
      }
    }
    if (nm == 0 || n < 3) continue;
    M3 R;
    double t[3], rmsd = 0.0;
    if (!rigid_fit(p, q, n, R, t, &rmsd) || rmsd > 0.5) continue;
    for (int m = 0; m < nm; ++m) {
      const int k = miss[m];
      const double tp3[3] = {tp.xyz[k][0], tp.xyz[k][1], tp.xyz[k][2]};
      for (int a = 0; a < 3; ++a)
        x[k * 3 + a] =
            static_cast<float>(R[a][0] * tp3[0] + R[a][1] * tp3[1] + R[a][2] * tp3[2] + t[a]);
      src[k] = kSrcInferred;
    }
  }
}

hkb_status load_text(std::string_view text, Format fmt, std::string_view origin,
                     const LoadOptions& opt, Structure* out) {
  std::vector<AtomRow> rows;
  hkb_status st = fmt == Format::kPdb ? parse_pdb(text, &rows) : parse_mmcif(text, &rows);
  if (st.code != HKB_OK) return st;
  if (rows.empty())
    return bad(fmt == Format::kPdb ? "no ATOM or HETATM records present in PDB input"
                                   : "no _atom_site rows present in mmCIF input");
  st = normalize(rows, opt, out);
  if (st.code != HKB_OK) return st;
  if (opt.infer_missing_atoms) infer_missing_atoms(out);
  out->origin = std::string(origin);
  return kOk;
}

// structure_loader.cpp:174-200: read, detect the format, parse.
hkb_status load_file(const std::string& path, const LoadOptions& opt, Structure* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return {HKB_UNAVAILABLE, "structure file not readable"};
  std::ostringstream buf;
  buf << f.rdbuf();
  const std::string text = buf.str();
  const Format fmt = detect_format(path, text);
  if (fmt == Format::kUnknown)
    return bad("unrecognized structure file format; extension and content cues did not match "
               "PDB or mmCIF");
  const size_t slash = path.find_last_of("/\\");
  return load_text(text, fmt, slash == std::string::npos ? path : path.substr(slash + 1), opt,
                   out);
}

}  // namespace hkb::io
