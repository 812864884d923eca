// Host-side decoding-order helpers shared by the engine and the C ABI.
#pragma once

#include <cstdint>

#include "hkb_mpnn.h"

namespace hkb {

std::uint64_t splitmix64_next(std::uint64_t& state);
double uniform01(std::uint64_t& state);
// Sort key of one residue: score (mask + 1e-4) |z|, ties by residue index.
struct OrderKey {
  float score;
  std::int32_t index;
};
// Random decoding order of L residues into `order`, using the caller's
// `keys` buffer of L entries as working storage (no allocation).
void random_decode_order_into(const float* mask, int L, std::uint64_t seed, OrderKey* keys,
                              std::int32_t* order);
// The same with its own working storage.
void random_decode_order(const float* mask, int L, std::uint64_t seed,
                         std::int32_t* order);
bool check_permutation(const std::int32_t* order, int L);

}  // namespace hkb
