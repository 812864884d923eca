// Seeded synthetic single-chain backbones for the benchmark configurations.
//
// Geometry: ideal N-CA-C-O chain placed atom by atom with the natural
// extension reference frame (NeRF) construction.  Bond lengths N-CA 1.458,
// CA-C 1.525, C-N 1.329, C=O 1.231 A; omega = 180 deg; Engh-Huber bond angles
// N-CA-C 111.2, CA-C-N 116.2, C-N-CA 121.7, CA-C=O 120.5 deg.  phi/psi come in
// runs of 4..12 residues: 60% helix (-57, -47) and 40% strand (-120, 130),
// jittered uniformly by +-10 deg (helix) or +-15 deg (strand).  O lies in the
// peptide plane trans to N(i+1).  The fifth slot is the virtual CB of the
// reference's structure input (cpp/io/virtual_cb.cpp:16-38; same coefficients)
// marked Virtual (3); every other atom is Observed (1).
//
// Randomness: std::mt19937_64 (fully specified by the C++ standard) with an
// explicit (x >> 11) * 2^-53 uniform transform, so the stream is the same on
// every conforming toolchain.

#include "hkb_mpnn.h"

#include <cmath>
#include <cstdint>
#include <random>
#include <vector>

namespace {

struct Vec3 {
  double x, y, z;
};
Vec3 sub(Vec3 a, Vec3 b) { return {a.x - b.x, a.y - b.y, a.z - b.z}; }
Vec3 add(Vec3 a, Vec3 b) { return {a.x + b.x, a.y + b.y, a.z + b.z}; }
Vec3 scale(Vec3 a, double s) { return {a.x * s, a.y * s, a.z * s}; }
Vec3 cross(Vec3 a, Vec3 b) {
  return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
Vec3 unit(Vec3 a) {
  const double n = std::sqrt(a.x * a.x + a.y * a.y + a.z * a.z);
  return scale(a, 1.0 / n);
}

constexpr double kDeg = 3.14159265358979323846 / 180.0;

// Place D so that |CD| = bond, angle(B,C,D) = angle, dihedral(A,B,C,D) = torsion.
Vec3 place(Vec3 a, Vec3 b, Vec3 c, double bond, double angle_deg,
           double torsion_deg) {
  const Vec3 bc = unit(sub(c, b));
  const Vec3 n = unit(cross(sub(b, a), bc));
  const Vec3 m = cross(n, bc);
  const double ang = angle_deg * kDeg, tor = torsion_deg * kDeg;
  const double d2x = -bond * std::cos(ang);
  const double d2y = bond * std::sin(ang) * std::cos(tor);
  const double d2z = bond * std::sin(ang) * std::sin(tor);
  return add(c, add(scale(bc, d2x), add(scale(m, d2y), scale(n, d2z))));
}

struct Stream {
  explicit Stream(std::uint64_t seed) : gen(seed) {}
  double uniform() { return static_cast<double>(gen() >> 11) * (1.0 / 9007199254740992.0); }
  std::mt19937_64 gen;
};

}  // namespace

extern "C" hkb_status hkb_synthetic_backbone(uint64_t seed, int32_t L,
                                             float* coords, uint8_t* sources) {
  if (L <= 0) return {HKB_INVALID_ARGUMENT, "synthetic backbone needs residue_count > 0"};
  if (coords == nullptr || sources == nullptr)
    return {HKB_INVALID_ARGUMENT, "synthetic backbone output pointers must be non-null"};
  Stream rng(seed);
  std::vector<double> phi(L), psi(L);
  int i = 0;
  while (i < L) {
    const bool helix = rng.uniform() < 0.6;
    const int run = 4 + static_cast<int>(rng.uniform() * 9.0);  // 4..12
    for (int r = 0; r < run && i < L; ++r, ++i) {
      const double j1 = 2.0 * rng.uniform() - 1.0, j2 = 2.0 * rng.uniform() - 1.0;
      if (helix) {
        phi[i] = -57.0 + 10.0 * j1;
        psi[i] = -47.0 + 10.0 * j2;
      } else {
        phi[i] = -120.0 + 15.0 * j1;
        psi[i] = 130.0 + 15.0 * j2;
      }
    }
  }
  constexpr double kNCa = 1.458, kCaC = 1.525, kCN = 1.329, kCO = 1.231;
  constexpr double kNCaC = 111.2, kCaCN = 116.2, kCNCa = 121.7, kCaCO = 120.5;
  std::vector<Vec3> N(L), CA(L), C(L), O(L);
  N[0] = {0.0, 0.0, 0.0};
  CA[0] = {kNCa, 0.0, 0.0};
  {
    const double a = (180.0 - kNCaC) * kDeg;
    C[0] = {kNCa + kCaC * std::cos(a), kCaC * std::sin(a), 0.0};
  }
  for (int r = 0; r + 1 < L; ++r) {
    N[r + 1] = place(N[r], CA[r], C[r], kCN, kCaCN, psi[r]);
    CA[r + 1] = place(CA[r], C[r], N[r + 1], kNCa, kCNCa, 180.0);
    C[r + 1] = place(C[r], N[r + 1], CA[r + 1], kCaC, kNCaC, phi[r + 1]);
  }
  for (int r = 0; r < L; ++r) O[r] = place(N[r], CA[r], C[r], kCO, kCaCO, psi[r] + 180.0);

  for (int r = 0; r < L; ++r) {
    const Vec3 at[4] = {N[r], CA[r], C[r], O[r]};
    for (int a = 0; a < 4; ++a) {
      coords[(r * 5 + a) * 3 + 0] = static_cast<float>(at[a].x);
      coords[(r * 5 + a) * 3 + 1] = static_cast<float>(at[a].y);
      coords[(r * 5 + a) * 3 + 2] = static_cast<float>(at[a].z);
      sources[r * 5 + a] = 1;
    }
    // Virtual CB in float arithmetic from the stored float N, CA, C.
    const float* n = coords + (r * 5 + 0) * 3;
    const float* ca = coords + (r * 5 + 1) * 3;
    const float* c = coords + (r * 5 + 2) * 3;
    const float b[3] = {ca[0] - n[0], ca[1] - n[1], ca[2] - n[2]};
    const float cv[3] = {c[0] - ca[0], c[1] - ca[1], c[2] - ca[2]};
    const float x[3] = {b[1] * cv[2] - b[2] * cv[1], b[2] * cv[0] - b[0] * cv[2],
                        b[0] * cv[1] - b[1] * cv[0]};
    for (int d = 0; d < 3; ++d)
      coords[(r * 5 + 4) * 3 + d] =
          ca[d] + -0.58273431F * x[d] + 0.56802827F * b[d] + -0.54067466F * cv[d];
    sources[r * 5 + 4] = 3;
  }
  return {HKB_OK, ""};
}
