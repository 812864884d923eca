// Minimal reader for the fp32 safetensors image of ProteinMPNN v_48_020:
// 8-byte little-endian header length, a JSON object mapping tensor names to
// {"dtype","shape","data_offsets"}, then the raw data.  Only F32 tensors are
// accepted (the reference weight file holds 118 of them).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace hkb {

struct TensorView {
  std::vector<int64_t> shape;
  const float* data = nullptr;  // points into the caller's buffer (may be unaligned-safe copy)
  int64_t count = 0;
};

// Parses `blob`; on failure returns false and sets *why to a static string.
bool parse_safetensors(const void* blob, size_t length,
                       std::map<std::string, TensorView>* out,
                       std::vector<float>* storage, const char** why);

}  // namespace hkb
