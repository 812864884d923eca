// Decoding orders on the host.
//
// The random order is ascending score_i = (mask_i + 1e-4) * |z_i| with z_i a
// Box-Muller normal from a SplitMix64 stream seeded by the sequence seed, ties
// broken by residue index (cpp/modules/mpnn/decode_order_scalar.cpp:21-42,
// 89-116).  It uses the host libm log/cos/sqrt in double precision, which is
// why it runs here and not on the device: the same glibc the reference links
// gives the same bits, and the device only consumes the resulting permutation.

#include "host_order.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

namespace hkb {

std::uint64_t splitmix64_next(std::uint64_t& state) {
  std::uint64_t z = (state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

double uniform01(std::uint64_t& state) {
  return static_cast<double>(splitmix64_next(state) >> 11) * (1.0 / 9007199254740992.0);
}

void random_decode_order_into(const float* mask, int L, std::uint64_t seed, OrderKey* keys,
                              std::int32_t* order) {
  std::uint64_t s = seed;
  for (int r = 0; r < L; ++r) {
    double u1 = uniform01(s);
    if (u1 <= 0.0) u1 = 1.0 / 9007199254740992.0;
    const double u2 = uniform01(s);
    const double radius = std::sqrt(-2.0 * std::log(u1));
    const float z = static_cast<float>(
        std::fabs(radius * std::cos(6.283185307179586476925286766559 * u2)));
    const float m = mask != nullptr ? mask[r] : 1.0F;
    keys[r] = {(m + 0.0001F) * z, r};
  }
  std::sort(keys, keys + L, [](const OrderKey& a, const OrderKey& b) {
    if (a.score != b.score) return a.score < b.score;
    return a.index < b.index;
  });
  for (int p = 0; p < L; ++p) order[p] = keys[p].index;
}

void random_decode_order(const float* mask, int L, std::uint64_t seed,
                         std::int32_t* order) {
  std::vector<OrderKey> keys(static_cast<std::size_t>(L));
  random_decode_order_into(mask, L, seed, keys.data(), order);
}

bool check_permutation(const std::int32_t* order, int L) {
  std::vector<unsigned char> seen(static_cast<std::size_t>(L), 0);
  for (int p = 0; p < L; ++p) {
    const std::int32_t r = order[p];
    if (r < 0 || r >= L || seen[r]) return false;
    seen[r] = 1;
  }
  return true;
}

}  // namespace hkb

extern "C" hkb_status hkb_mpnn_decode_order(int32_t L, const float* mask,
                                            uint64_t seed, int32_t mode,
                                            const int32_t* input_order,
                                            int32_t* order) {
  if (L < 0) return {HKB_INVALID_ARGUMENT, "residue_count must be >= 0"};
  if (L > 0 && order == nullptr)
    return {HKB_INVALID_ARGUMENT, "ProteinMPNN decode order output pointer is null"};
  switch (mode) {
    case HKB_DECODE_RANDOM:
      hkb::random_decode_order(mask, L, seed, order);
      return {HKB_OK, ""};
    case HKB_DECODE_N_TO_C:
      for (int p = 0; p < L; ++p) order[p] = p;
      return {HKB_OK, ""};
    case HKB_DECODE_INPUT:
      if (input_order == nullptr && L > 0)
        return {HKB_INVALID_ARGUMENT, "ProteinMPNN input decoding_order must be a permutation"};
      if (!hkb::check_permutation(input_order, L))
        return {HKB_INVALID_ARGUMENT, "ProteinMPNN input decoding_order must be a permutation"};
      for (int p = 0; p < L; ++p) order[p] = input_order[p];
      return {HKB_OK, ""};
    default:
      return {HKB_INVALID_ARGUMENT, "unknown decode order mode"};
  }
}
