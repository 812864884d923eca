// Engine internals shared by the C ABI (engine.cu) and the bf16 path.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "hkb_mpnn.h"
#include "kernels.hpp"

namespace hkb {

// Capacity of the device decoding-order kernel's recheck list.
constexpr int kRecheckCap = 255;

// Named, grow-only device buffers reused across calls.
class Workspace {
 public:
  ~Workspace() { release(); }
  void* get(const std::string& name, size_t bytes);
  template <typename T>
  T* get_as(const std::string& name, size_t count) {
    return static_cast<T*>(get(name, count * sizeof(T)));
  }
  void release();
  size_t bytes() const;

 private:
  struct Buf {
    void* p = nullptr;
    size_t n = 0;
  };
  std::map<std::string, Buf> bufs_;
};

// Host-side description of one validated batch.
struct HostBatch {
  int B = 0;
  int R = 0;
  int64_t Q = 0;
  int NS = 0;
  int max_len = 0;
  std::vector<int> L, off, S, seq_base;
  std::vector<int64_t> qoff;          // [B] first row of protein b
  std::vector<int> res_prot;          // [R]
  std::vector<int> seq_prot;          // [NS]
  std::vector<int64_t> seq_row_off;   // [NS]
  std::vector<uint64_t> seq_seed;     // [NS]
  std::vector<float> seq_temp;        // [NS]
  std::vector<float> mask;            // [R]
  std::vector<int32_t> orders;        // [Q]
};

// Device copies of the per-batch tables + BatchView pointing at them.
struct DeviceBatch {
  BatchView bv;
  const float* coords = nullptr;
  const uint8_t* sources = nullptr;
};

struct EncoderOut {
  int* e_idx = nullptr;   // [R,48]
  float* d2 = nullptr;    // [R,48]
  float* mask = nullptr;  // [R]
  float* h_e = nullptr;   // [R,48,128] (fp32 encoder)
  uint16_t* h_e16 = nullptr;  // [h_e_rows,128] fp16 (tensor-core encoder); rows past R*48 are 0
  uint16_t* h_e16lo = nullptr;  // [R*48,128] its fp16 remainder (h_E = hi + lo)
  int64_t h_e_rows = 0;         // rows of h_e16: max(R*48, one TMA box of the encoder passes)
  float* h_v = nullptr;   // [R,128]
};

}  // namespace hkb

struct hkb_engine {
  int device = 0;
  int precision = HKB_PRECISION_FP32;
  cudaStream_t stream = nullptr;
  void* d_weights = nullptr;
  size_t weights_bytes = 0;
  hkb::F32Weights w32{};
  void* d_stream = nullptr;          // 16-bit decode weight tiles (SW128 images)
  hkb::Bf16DecodeWeights wbf{};
  void* d_gemm = nullptr;            // fp16 GEMM weight images (tensor-core modes)
  void* d_head = nullptr;            // decode kernel's logit head [21][kHeadPitch]
  std::map<std::string, const unsigned char*> gemm_img;
  int num_sms = 148;
  hkb::Workspace ws;
  unsigned int* d_err = nullptr;
  int64_t launches = 0;
  float timings[4] = {0, 0, 0, 0};
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // pinned staging of the host-generated decoding orders; ev_orders marks the
  // last upload from it, so the next call does not overwrite it in flight
  int32_t* h_orders = nullptr;
  size_t h_orders_cap = 0;
  cudaEvent_t ev_orders = nullptr;
  // device decoding orders: pinned read-back of the recheck count and list
  // ([0] count, then up to kRecheckCap sequence indices), its event, and the
  // number of sequences the host has recomputed so far
  unsigned int* h_recheck = nullptr;
  cudaEvent_t ev_recheck = nullptr;
  int recheck_all_orders = 0;
  int stall_check_calls = 0;   // test hook: decode calls that run the failure-path check
  int64_t orders_rechecked = 0;
};
