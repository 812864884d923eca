// `hikoboshi design` command-line tool on the B200 engine: same flags,
// defaults, diagnostics, exit codes and output files as the reference's
// (cli/commands/design.cpp:52-356, cli/options.cpp, cli/exit_codes.cpp,
// cli/weights_resolution.cpp).  Extra flags of this build: --precision
// fp32|f16 (default fp32, the reference's arithmetic) and --device N.  The
// weights are the safetensors image beside the library
// (../weights/Hikoboshi-ProteinMPNN-v48-020.safetensors relative to this
// binary) unless HKB_MPNN_WEIGHTS names another file.
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <limits>
#include <string>
#include <string_view>

#include "hkb_design_api.hpp"

namespace {

using hikoboshi::universal::Status;

constexpr Status kOk{HKB_OK, ""};
Status invalid(const char* d) { return {HKB_INVALID_ARGUMENT, d}; }

const char* code_name(int32_t c) {
  switch (c) {
    case HKB_OK: return "ok";
    case HKB_INVALID_ARGUMENT: return "invalid_argument";
    case HKB_FAILED_PRECONDITION: return "failed_precondition";
    case HKB_UNAVAILABLE: return "unavailable";
    case HKB_UNIMPLEMENTED: return "unimplemented";
    case HKB_INTERNAL_ERROR: return "internal_error";
  }
  return "unknown_status";
}

// Exit codes: 0 ok, 2 invalid argument / failed precondition, 3 I/O
// unavailable, 4 unimplemented, 5 internal failure; the message goes to stderr
// as "hikoboshi: <code>[: <detail>]".
int report(Status s) {
  if (s.code == HKB_OK) return 0;
  std::cerr << "hikoboshi: " << code_name(s.code);
  if (s.detail && s.detail[0]) std::cerr << ": " << s.detail;
  std::cerr << '\n';
  switch (s.code) {
    case HKB_INVALID_ARGUMENT:
    case HKB_FAILED_PRECONDITION: return 2;
    case HKB_UNAVAILABLE: return 3;
    case HKB_UNIMPLEMENTED: return 4;
    default: return 5;
  }
}

bool nocase_eq(std::string_view a, std::string_view b) {
  if (a.size() != b.size()) return false;
  for (size_t i = 0; i < a.size(); ++i) {
    char x = a[i], y = b[i];
    if (x >= 'A' && x <= 'Z') x = static_cast<char>(x + 32);
    if (y >= 'A' && y <= 'Z') y = static_cast<char>(y + 32);
    if (x != y) return false;
  }
  return true;
}

bool ends_nocase(std::string_view v, std::string_view suf) {
  return v.size() >= suf.size() && nocase_eq(v.substr(v.size() - suf.size()), suf);
}

// `--name=value` assignment form.
bool assignment(std::string_view arg, std::string_view name, std::string* value) {
  if (arg.size() <= name.size() + 1 || arg.substr(0, name.size()) != name ||
      arg[name.size()] != '=')
    return false;
  *value = std::string(arg.substr(name.size() + 1));
  return true;
}

bool historical_flag(std::string_view a) {
  for (const char* f : {"--soft", "--soft-sw", "--temperature", "--anneal", "--save-frames",
                        "--tree", "--msa", "--database", "--gpu", "--simd"})
    if (a == f) return true;
  return false;
}

bool parse_float(const std::string& t, float* v) {
  char* end = nullptr;
  errno = 0;
  const float x = std::strtof(t.c_str(), &end);
  if (errno != 0 || end == t.c_str() || *end != '\0') return false;
  *v = x;
  return true;
}

bool parse_u64(const std::string& t, unsigned long long* v) {
  char* end = nullptr;
  errno = 0;
  const unsigned long long x = std::strtoull(t.c_str(), &end, 10);
  if (errno != 0 || end == t.c_str() || *end != '\0') return false;
  *v = x;
  return true;
}

constexpr const char* kPackageList =
    "hikoboshi-mpnn-d64, mpnn64, mpnn-64, Hikoboshi-MPNN-64, hikoboshi-esm2-8m, esm2-8m, "
    "esm2_8m, Hikoboshi-ESM2-8M, proteinmpnn-v48-eps020, v_48_020, "
    "Hikoboshi-ProteinMPNN-v48-020, proteinmpnn-v48-020, proteinmpnn";

// Package names of the reference's registry.  Only the ProteinMPNN package
// runs design; the others resolve and then fail in inverse_fold, as there.
enum class Package { kUnknown, kProteinMpnn, kOther };

Package classify_package(std::string_view v, const char** canonical) {
  static const char* kMpnn[] = {"proteinmpnn-v48-eps020", "v_48_020",
                                "Hikoboshi-ProteinMPNN-v48-020", "proteinmpnn-v48-020",
                                "proteinmpnn"};
  static const char* kD64[] = {"hikoboshi-mpnn-d64", "mpnn64", "mpnn-64", "Hikoboshi-MPNN-64"};
  static const char* kEsm[] = {"hikoboshi-esm2-8m", "esm2-8m", "esm2_8m", "Hikoboshi-ESM2-8M"};
  for (const char* n : kMpnn)
    if (nocase_eq(v, n)) return *canonical = kMpnn[0], Package::kProteinMpnn;
  for (const char* n : kD64)
    if (nocase_eq(v, n)) return *canonical = kD64[0], Package::kOther;
  for (const char* n : kEsm)
    if (nocase_eq(v, n)) return *canonical = kEsm[0], Package::kOther;
  return Package::kUnknown;
}

bool file_like(std::string_view v) {
  if (v.find('/') != std::string_view::npos || v.find('\\') != std::string_view::npos) return true;
  for (const char* s : {".bin", ".ckpt", ".dat", ".gz", ".h5", ".hdf5", ".json", ".model", ".npy",
                        ".npz", ".onnx", ".pb", ".pickle", ".pkg", ".pkl", ".pt", ".pth",
                        ".safetensors", ".tar", ".tar.gz", ".tgz", ".toml", ".txt", ".weights",
                        ".yaml", ".yml", ".zip"})
    if (ends_nocase(v, s)) return true;
  return false;
}

struct Options {
  std::string pdb, out, out_logprobs;
  std::string package_id = "proteinmpnn-v48-eps020";
  Package package = Package::kProteinMpnn;
  float sampling_temp = 0.1f;
  unsigned long long num_seqs = 1, seed = 0;
  hikoboshi::api::InverseFoldDecodeOrder order = hikoboshi::api::InverseFoldDecodeOrder::Random;
  float backbone_noise = 0.0f;
  int32_t precision = HKB_PRECISION_FP32;
  int device = 0;
};

void usage(std::ostream& out) {
  out << "usage: hikoboshi design --pdb INPUT.pdb --out OUT.fasta [options]\n"
      << "\n"
      << "options:\n"
      << "  --num-seqs N             number of sequences to design (default 1)\n"
      << "  --sampling-temp T        sampling temperature (default 0.1)\n"
      << "  --seed N                 deterministic sampling seed (default 0)\n"
      << "  --decode-order random|n_to_c\n"
      << "  --package NAME           compiled ProteinMPNN package ID or alias\n"
      << "  --backbone-noise SIGMA   coordinate noise sigma (default 0.0)\n"
      << "  --out-logprobs PATH      write opt-in [N,L,21] log-prob NPZ\n"
      << "  --precision fp32|f16     engine arithmetic (default fp32)\n"
      << "  --device N               CUDA device (default 0)\n";
}

Status resolve_package(const std::string& v, Options* o) {
  if (file_like(v)) {
    static const std::string msg =
        std::string("external package paths are not supported in Hikoboshi 0.1.0; use a "
                    "compiled package ID or alias: ") + kPackageList;
    return invalid(msg.c_str());
  }
  const char* canonical = nullptr;
  const Package p = classify_package(v, &canonical);
  if (p == Package::kUnknown) {
    static const std::string msg =
        std::string("unknown Hikoboshi package id; available compiled package IDs/aliases: ") +
        kPackageList;
    return invalid(msg.c_str());
  }
  if (v != canonical)
    std::fprintf(stderr, "warning: package alias '%s' is deprecated; use '%s'\n", v.c_str(),
                 canonical);
  o->package = p;
  o->package_id = v;
  return kOk;
}

Status parse(int argc, char** argv, Options* o) {
  for (int i = 0; i < argc; ++i) {
    const std::string_view arg(argv[i]);
    if (historical_flag(arg))
      return invalid("that historical or reserved flag is not available in Hikoboshi 0.1.0");
    std::string value;
    // value of `--name VALUE` or `--name=VALUE`; false if this is not --name
    auto take = [&](const char* name, Status* st) {
      if (!assignment(arg, name, &value) && arg != name) return false;
      if (value.empty()) {
        if (i + 1 >= argc) {
          *st = invalid("option requires a value");
          return true;
        }
        value = argv[++i];
      }
      *st = kOk;
      return true;
    };
    Status st = kOk;
    if (take("--package", &st)) {
      if (st.code != HKB_OK) return st;
      st = resolve_package(value, o);
      if (st.code != HKB_OK) return st;
      continue;
    }
    for (const char* n : {"--external-package", "--package-path", "--weights"}) {
      std::string ignored;
      if (arg == n || assignment(arg, n, &ignored))
        return invalid("external package paths are not supported in Hikoboshi 0.1.0; design "
                       "uses the compiled ProteinMPNN registered package");
    }
    if (take("--pdb", &st)) {
      if (st.code != HKB_OK) return st;
      o->pdb = value;
    } else if (take("--out", &st)) {
      if (st.code != HKB_OK) return st;
      o->out = value;
    } else if (take("--out-logprobs", &st)) {
      if (st.code != HKB_OK) return st;
      o->out_logprobs = value;
    } else if (take("--sampling-temp", &st)) {
      if (st.code != HKB_OK) return st;
      if (!parse_float(value, &o->sampling_temp))
        return invalid("sampling-temp must be a finite number");
    } else if (take("--backbone-noise", &st)) {
      if (st.code != HKB_OK) return st;
      if (!parse_float(value, &o->backbone_noise))
        return invalid("backbone-noise must be a finite number");
    } else if (take("--num-seqs", &st)) {
      if (st.code != HKB_OK) return st;
      if (!parse_u64(value, &o->num_seqs) || o->num_seqs == 0)
        return invalid("num-seqs must be a positive integer");
    } else if (take("--seed", &st)) {
      if (st.code != HKB_OK) return st;
      if (!parse_u64(value, &o->seed)) return invalid("seed must be a non-negative integer");
    } else if (take("--decode-order", &st)) {
      if (st.code != HKB_OK) return st;
      if (value == "random") o->order = hikoboshi::api::InverseFoldDecodeOrder::Random;
      else if (value == "n_to_c" || value == "n-to-c")
        o->order = hikoboshi::api::InverseFoldDecodeOrder::NToC;
      else return invalid("decode-order must be random or n_to_c");
    } else if (take("--precision", &st)) {
      if (st.code != HKB_OK) return st;
      if (value == "fp32") o->precision = HKB_PRECISION_FP32;
      else if (value == "f16") o->precision = HKB_PRECISION_F16;
      else return invalid("precision must be fp32 or f16");
    } else if (take("--device", &st)) {
      if (st.code != HKB_OK) return st;
      unsigned long long d = 0;
      if (!parse_u64(value, &d) || d > 1024) return invalid("device must be a CUDA device ordinal");
      o->device = static_cast<int>(d);
    } else if (!arg.empty() && arg.front() == '-') {
      return invalid("unknown design option");
    } else {
      return invalid("design requires explicit --pdb and --out options");
    }
  }
  if (o->pdb.empty()) return invalid("design requires --pdb");
  if (o->out.empty()) return invalid("design requires --out");
  return kOk;
}

std::string default_weights() {
  if (const char* env = std::getenv("HKB_MPNN_WEIGHTS")) return env;
  char buf[4096];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof(buf) - 1);
  std::string dir = n > 0 ? std::string(buf, (size_t)n) : std::string(".");
  dir = dir.substr(0, dir.find_last_of('/'));
  return dir + "/../weights/Hikoboshi-ProteinMPNN-v48-020.safetensors";
}

int run_design(int argc, char** argv) {
  if (argc > 0 && (std::string_view(argv[0]) == "-h" || std::string_view(argv[0]) == "--help")) {
    usage(std::cout);
    return 0;
  }
  Options o;
  Status st = parse(argc, argv, &o);
  if (st.code != HKB_OK) return report(st);
  const auto loaded = hikoboshi::io::load_structure_from_file(o.pdb);
  if (loaded.status.code != HKB_OK) return report(loaded.status);
  const auto engine = hikoboshi::api::Engine::create(default_weights(), o.device, o.precision);
  if (engine.status.code != HKB_OK) return report(engine.status);
  if (o.package != Package::kProteinMpnn)
    return report(invalid("inverse_fold requires proteinmpnn-v48-eps020; it does not use the "
                          "aligner hikoboshi-mpnn-d64 package"));
  hikoboshi::api::InverseFoldRequest rq;
  const auto& s = loaded.value;
  rq.structure = {static_cast<size_t>(s.residue_count()), s.coordinates().data(),
                  s.atom_sources().data(), s.residue_codes().data()};
  rq.pdb_path = o.pdb;
  rq.package = o.package_id;
  rq.sampling_temp = o.sampling_temp;
  rq.num_seqs = static_cast<size_t>(o.num_seqs);
  rq.seed = o.seed;
  rq.decode_order = o.order;
  rq.backbone_noise = o.backbone_noise;
  rq.logprobs_out = o.out_logprobs;
  const auto result = engine.value.inverse_fold(rq);
  if (result.status.code != HKB_OK) return report(result.status);
  hikoboshi::io::DesignFastaWriterOptions wo;
  wo.sampling_temp = o.sampling_temp;
  st = hikoboshi::io::write_design_fasta(o.out, result.value, wo);
  if (st.code != HKB_OK) return report(st);
  if (!o.out_logprobs.empty()) {
    st = hikoboshi::io::write_inverse_fold_logprobs_npz(o.out_logprobs, result.value);
    if (st.code != HKB_OK) return report(st);
  }
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2 || std::string_view(argv[1]) == "-h" || std::string_view(argv[1]) == "--help") {
    std::cout << "usage: hikoboshi design --pdb INPUT.pdb --out OUT.fasta [options]\n";
    return argc < 2 ? 2 : 0;
  }
  if (std::string_view(argv[1]) != "design")
    return report(invalid("this build provides the design command only"));
  return run_design(argc - 2, argv + 2);
}
