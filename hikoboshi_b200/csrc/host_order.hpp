// Host-side decoding-order helpers shared by the engine and the C ABI.
#pragma once

#include <cstdint>

#include "hkb_mpnn.h"

namespace hkb {

std::uint64_t splitmix64_next(std::uint64_t& state);
double uniform01(std::uint64_t& state);
void random_decode_order(const float* mask, int L, std::uint64_t seed,
                         std::int32_t* order);
bool check_permutation(const std::int32_t* order, int L);

}  // namespace hkb
