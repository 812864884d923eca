// C ABI of the ProteinMPNN v_48_020 design engine: weight binding, batch
// validation, decoding orders, and the device pipeline
//   kNN -> edge features -> edge embedding -> 3 encoder layers
//   -> decoder tables -> fused autoregressive decode (or teacher-forced pass).
#include "engine.hpp"
#include "common.cuh"

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <numeric>
#include <thread>

#include <sched.h>

#include <nvtx3/nvToolsExt.h>

#include "host_order.hpp"
#include "safetensors.hpp"

namespace hkb {

void* Workspace::get(const std::string& name, size_t bytes) {
  Buf& b = bufs_[name];
  if (bytes == 0) bytes = 16;
  if (b.n < bytes) {
    if (b.p) cudaFree(b.p);
    b.p = nullptr;
    b.n = 0;
    const size_t want = bytes + bytes / 8;  // slack against small growth
    if (cudaMalloc(&b.p, want) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    b.n = want;
  }
  return b.p;
}

void Workspace::release() {
  for (auto& kv : bufs_)
    if (kv.second.p) cudaFree(kv.second.p);
  bufs_.clear();
}

size_t Workspace::bytes() const {
  size_t t = 0;
  for (const auto& kv : bufs_) t += kv.second.n;
  return t;
}

namespace {

constexpr hkb_status kOk{HKB_OK, ""};

// NVTX range over the host-side enqueue of one pipeline phase (featurise +
// encode, decoder tables, decode / teacher-forced layers): profilers show it
// on the CPU timeline and correlate it with the phase's kernels.  Costs
// nothing unless a tool is attached.
struct PhaseRange {
  explicit PhaseRange(const char* name) { nvtxRangePushA(name); }
  ~PhaseRange() { nvtxRangePop(); }
  PhaseRange(const PhaseRange&) = delete;
  PhaseRange& operator=(const PhaseRange&) = delete;
};

hkb_status invalid(const char* d) { return {HKB_INVALID_ARGUMENT, d}; }
hkb_status internal(const char* d) { return {HKB_INTERNAL_ERROR, d}; }

#define HKB_CUDA(call)                                                   \
  do {                                                                   \
    cudaError_t e_ = (call);                                             \
    if (e_ != cudaSuccess) return {HKB_INTERNAL_ERROR, cudaGetErrorString(e_)}; \
  } while (0)

// --------------------------------------------------------------------------
// Weight binding and re-layout
// --------------------------------------------------------------------------
struct Blob {
  std::vector<float> data;
  size_t add(const float* src, size_t n) {
    const size_t at = (data.size() + 63) / 64 * 64;  // 256-byte aligned
    data.resize(at + n);
    if (src) std::memcpy(data.data() + at, src, n * sizeof(float));
    return at;
  }
  size_t add_zero(size_t n) { return add(nullptr, n); }
};

// out[i*rows + o] = W[o*cols + i] for W [rows=out, cols=in] restricted to
// input columns [c0, c0+width): the [in][out] layout the SIMT kernels read.
void transpose_block(const float* W, int out_dim, int in_dim, int c0, int width,
                     float* dst, int ld_dst, int dst_col0) {
  for (int i = 0; i < width; ++i)
    for (int o = 0; o < out_dim; ++o)
      dst[(size_t)i * ld_dst + dst_col0 + o] = W[(size_t)o * in_dim + c0 + i];
}

struct Prepared {
  Blob blob;
  // offsets of each field, resolved to device pointers after upload
  std::map<std::string, size_t> at;
};

bool get_tensor(const std::map<std::string, TensorView>& t, const std::string& name,
                std::vector<int64_t> shape, const float** out) {
  auto it = t.find(name);
  if (it == t.end()) return false;
  if (it->second.shape != shape) return false;
  *out = it->second.data;
  return true;
}

hkb_status prepare_f32(const std::map<std::string, TensorView>& t, Prepared* P) {
  auto& B = P->blob;
  auto& at = P->at;
  const float* x = nullptr;
  auto need = [&](const std::string& n, std::vector<int64_t> s) -> const float* {
    const float* p = nullptr;
    if (!get_tensor(t, n, s, &p)) return nullptr;
    return p;
  };
  if (t.size() != 118) return invalid("ProteinMPNN v_48_020 weights must hold 118 tensors");
  if (!(x = need("features.embeddings.linear.weight", {16, 66}))) goto bad;
  at["pos_w"] = B.add(x, 16 * 66);
  if (!(x = need("features.embeddings.linear.bias", {16}))) goto bad;
  at["pos_b"] = B.add(x, 16);
  if (!(x = need("features.edge_embedding.weight", {128, 416}))) goto bad;
  at["edge_wT"] = B.add_zero(416 * 128);
  transpose_block(x, 128, 416, 0, 416, B.data.data() + at["edge_wT"], 128, 0);
  if (!(x = need("features.norm_edges.weight", {128}))) goto bad;
  at["norm_e_w"] = B.add(x, 128);
  if (!(x = need("features.norm_edges.bias", {128}))) goto bad;
  at["norm_e_b"] = B.add(x, 128);
  if (!(x = need("W_e.weight", {128, 128}))) goto bad;
  at["We_T"] = B.add_zero(128 * 128);
  transpose_block(x, 128, 128, 0, 128, B.data.data() + at["We_T"], 128, 0);
  if (!(x = need("W_e.bias", {128}))) goto bad;
  at["We_b"] = B.add(x, 128);
  {
    const float* Ws = need("W_s.weight", {21, 128});
    if (!Ws) goto bad;
    for (int l = 0; l < 3; ++l) {
      const std::string p = "encoder_layers." + std::to_string(l) + ".";
      const std::string q = "enc" + std::to_string(l) + ".";
      for (const char* nm : {"W1", "W11"}) {
        const float* W = need(p + nm + ".weight", {128, 384});
        const float* bb = need(p + nm + ".bias", {128});
        if (!W || !bb) goto bad;
        const std::string key = q + nm;
        at[key + "acT"] = B.add_zero(128 * 256);
        float* dst = B.data.data() + at[key + "acT"];
        transpose_block(W, 128, 384, 0, 128, dst, 256, 0);    // h_i block
        transpose_block(W, 128, 384, 256, 128, dst, 256, 128); // h_j block
        at[key + "bT"] = B.add_zero(128 * 128);
        transpose_block(W, 128, 384, 128, 128, B.data.data() + at[key + "bT"], 128, 0);
        at[key + "b_ac"] = B.add_zero(256);
        std::memcpy(B.data.data() + at[key + "b_ac"], bb, 128 * sizeof(float));
      }
      for (const char* nm : {"W2", "W3", "W12", "W13"}) {
        const float* W = need(p + nm + ".weight", {128, 128});
        const float* bb = need(p + nm + ".bias", {128});
        if (!W || !bb) goto bad;
        at[q + nm + "T"] = B.add_zero(128 * 128);
        transpose_block(W, 128, 128, 0, 128, B.data.data() + at[q + nm + "T"], 128, 0);
        at[q + nm + "b"] = B.add(bb, 128);
      }
      for (const char* nm : {"norm1", "norm2", "norm3"}) {
        const float* g = need(p + nm + ".weight", {128});
        const float* bb = need(p + nm + ".bias", {128});
        if (!g || !bb) goto bad;
        at[q + nm + "w"] = B.add(g, 128);
        at[q + nm + "b"] = B.add(bb, 128);
      }
      {
        const float* Wi = need(p + "dense.W_in.weight", {512, 128});
        const float* bi = need(p + "dense.W_in.bias", {512});
        const float* Wo = need(p + "dense.W_out.weight", {128, 512});
        const float* bo = need(p + "dense.W_out.bias", {128});
        if (!Wi || !bi || !Wo || !bo) goto bad;
        at[q + "WinT"] = B.add_zero(128 * 512);
        transpose_block(Wi, 512, 128, 0, 128, B.data.data() + at[q + "WinT"], 512, 0);
        at[q + "bin"] = B.add(bi, 512);
        at[q + "WoutT"] = B.add_zero(512 * 128);
        transpose_block(Wo, 128, 512, 0, 512, B.data.data() + at[q + "WoutT"], 128, 0);
        at[q + "bout"] = B.add(bo, 128);
      }
    }
    for (int l = 0; l < 3; ++l) {
      const std::string p = "decoder_layers." + std::to_string(l) + ".";
      const std::string q = "dec" + std::to_string(l) + ".";
      const float* W = need(p + "W1.weight", {128, 512});
      const float* b1 = need(p + "W1.bias", {128});
      if (!W || !b1) goto bad;
      // input blocks of the decoder W1: [h_t | h_E | h_S_j | h_j]
      at[q + "W1adT"] = B.add_zero(128 * 256);
      transpose_block(W, 128, 512, 0, 128, B.data.data() + at[q + "W1adT"], 256, 0);
      transpose_block(W, 128, 512, 384, 128, B.data.data() + at[q + "W1adT"], 256, 128);
      at[q + "b1ad"] = B.add_zero(256);
      std::memcpy(B.data.data() + at[q + "b1ad"], b1, 128 * sizeof(float));
      at[q + "W1aT"] = B.add_zero(128 * 128);
      transpose_block(W, 128, 512, 0, 128, B.data.data() + at[q + "W1aT"], 128, 0);
      at[q + "b1"] = B.add(b1, 128);
      at[q + "W1dT"] = B.add_zero(128 * 128);
      transpose_block(W, 128, 512, 384, 128, B.data.data() + at[q + "W1dT"], 128, 0);
      at[q + "W1bT"] = B.add_zero(128 * 128);
      transpose_block(W, 128, 512, 128, 128, B.data.data() + at[q + "W1bT"], 128, 0);
      // Stab[v][o] = sum_i W1c[o][i] W_s[v][i]: the sequence-embedding term
      // of every neighbour slot is one of 21 vectors per layer.
      at[q + "Stab"] = B.add_zero(21 * 128);
      for (int v = 0; v < 21; ++v)
        for (int o = 0; o < 128; ++o) {
          double acc = 0.0;
          for (int i = 0; i < 128; ++i)
            acc += (double)W[(size_t)o * 512 + 256 + i] * (double)Ws[(size_t)v * 128 + i];
          B.data[at[q + "Stab"] + (size_t)v * 128 + o] = (float)acc;
        }
      for (const char* nm : {"W2", "W3"}) {
        const float* Wm = need(p + nm + ".weight", {128, 128});
        const float* bb = need(p + nm + ".bias", {128});
        if (!Wm || !bb) goto bad;
        at[q + nm + "T"] = B.add_zero(128 * 128);
        transpose_block(Wm, 128, 128, 0, 128, B.data.data() + at[q + nm + "T"], 128, 0);
        at[q + nm + "b"] = B.add(bb, 128);
      }
      for (const char* nm : {"norm1", "norm2"}) {
        const float* g = need(p + nm + ".weight", {128});
        const float* bb = need(p + nm + ".bias", {128});
        if (!g || !bb) goto bad;
        at[q + nm + "w"] = B.add(g, 128);
        at[q + nm + "b"] = B.add(bb, 128);
      }
      const float* Wi = need(p + "dense.W_in.weight", {512, 128});
      const float* bi = need(p + "dense.W_in.bias", {512});
      const float* Wo = need(p + "dense.W_out.weight", {128, 512});
      const float* bo = need(p + "dense.W_out.bias", {128});
      if (!Wi || !bi || !Wo || !bo) goto bad;
      at[q + "WinT"] = B.add_zero(128 * 512);
      transpose_block(Wi, 512, 128, 0, 128, B.data.data() + at[q + "WinT"], 512, 0);
      at[q + "bin"] = B.add(bi, 512);
      at[q + "WoutT"] = B.add_zero(512 * 128);
      transpose_block(Wo, 128, 512, 0, 512, B.data.data() + at[q + "WoutT"], 128, 0);
      at[q + "bout"] = B.add(bo, 128);
    }
  }
  if (!(x = need("W_out.weight", {21, 128}))) goto bad;
  at["headT"] = B.add_zero(128 * 21);
  transpose_block(x, 21, 128, 0, 128, B.data.data() + at["headT"], 21, 0);
  if (!(x = need("W_out.bias", {21}))) goto bad;
  at["head_b"] = B.add(x, 21);
  return kOk;
bad:
  return invalid("ProteinMPNN v_48_020 weights: missing tensor or wrong shape");
}

void resolve_f32(const Prepared& P, const float* base, F32Weights* w) {
  auto f = [&](const std::string& k) { return base + P.at.at(k); };
  w->pos_w = f("pos_w");
  w->pos_b = f("pos_b");
  w->edge_wT = f("edge_wT");
  w->norm_e_w = f("norm_e_w");
  w->norm_e_b = f("norm_e_b");
  w->We_T = f("We_T");
  w->We_b = f("We_b");
  for (int l = 0; l < 3; ++l) {
    const std::string q = "enc" + std::to_string(l) + ".";
    auto& E = w->enc[l];
    E.W1acT = f(q + "W1acT");
    E.b1ac = f(q + "W1b_ac");
    E.W1bT = f(q + "W1bT");
    E.W11acT = f(q + "W11acT");
    E.b11ac = f(q + "W11b_ac");
    E.W11bT = f(q + "W11bT");
    E.W2T = f(q + "W2T");
    E.b2 = f(q + "W2b");
    E.W3T = f(q + "W3T");
    E.b3 = f(q + "W3b");
    E.W12T = f(q + "W12T");
    E.b12 = f(q + "W12b");
    E.W13T = f(q + "W13T");
    E.b13 = f(q + "W13b");
    E.n1w = f(q + "norm1w");
    E.n1b = f(q + "norm1b");
    E.n2w = f(q + "norm2w");
    E.n2b = f(q + "norm2b");
    E.n3w = f(q + "norm3w");
    E.n3b = f(q + "norm3b");
    E.WinT = f(q + "WinT");
    E.bin = f(q + "bin");
    E.WoutT = f(q + "WoutT");
    E.bout = f(q + "bout");
  }
  for (int l = 0; l < 3; ++l) {
    const std::string q = "dec" + std::to_string(l) + ".";
    auto& D = w->dec[l];
    D.W1adT = f(q + "W1adT");
    D.b1ad = f(q + "b1ad");
    D.W1aT = f(q + "W1aT");
    D.b1 = f(q + "b1");
    D.W1dT = f(q + "W1dT");
    D.W1bT = f(q + "W1bT");
    D.Stab = f(q + "Stab");
    D.W2T = f(q + "W2T");
    D.b2 = f(q + "W2b");
    D.W3T = f(q + "W3T");
    D.b3 = f(q + "W3b");
    D.n1w = f(q + "norm1w");
    D.n1b = f(q + "norm1b");
    D.n2w = f(q + "norm2w");
    D.n2b = f(q + "norm2b");
    D.WinT = f(q + "WinT");
    D.bin = f(q + "bin");
    D.WoutT = f(q + "WoutT");
    D.bout = f(q + "bout");
  }
  w->headT = f("headT");
  w->head_b = f("head_b");
}

// --------------------------------------------------------------------------
// 16-bit decode weight stream: kStreamTilesPerStep SW128 tile images in
// consumption order
// --------------------------------------------------------------------------
uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return (uint16_t)((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  u += 0x7FFFu + ((u >> 16) & 1u);   // round to nearest even
  return (uint16_t)(u >> 16);
}

// IEEE binary16, round to nearest even (overflow to inf, gradual underflow).
uint16_t f2h(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t e8 = (x >> 23) & 0xFFu;
  uint32_t mant = x & 0x7FFFFFu;
  if (e8 == 0xFFu) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0u));
  const int exp = (int)e8 - 127 + 15;
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    const int shift = 14 - exp;
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = sign | ((uint32_t)exp << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)h;
}

// IEEE binary16 -> binary32 (exact).
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0) {
    if (man == 0) {
      bits = sign;
    } else {   // subnormal: renormalise
      ex = 113;
      while (!(man & 0x400u)) {
        man <<= 1;
        --ex;
      }
      bits = sign | (ex << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (ex == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((ex + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// bf16 -> fp32 (exact).
float bf_to_float(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// The 16-bit rounding of v, or (lo) the 16-bit rounding of its remainder
// v - hi: W = hi + lo carries about twice the 16-bit precision, and a product
// W x is formed as hi x + lo x by two MMAs into one fp32 accumulator.
uint16_t to16(float v, bool f16, bool lo) {
  const uint16_t hi = f16 ? f2h(v) : f2bf(v);
  if (!lo) return hi;
  const float r = v - (f16 ? half_to_float(hi) : bf_to_float(hi));   // exact in fp32
  return f16 ? f2h(r) : f2bf(r);
}

bool g_tile_f16 = true;   // operand format of the tiles being appended

// Image of the 128 x 128 block W[r0:r0+128, k0:k0+128] (W row-major with
// leading dimension ld) in the SW128 K-major layout of tcgen05.cuh.
void append_tile(std::vector<uint16_t>& img, const float* W, int ld, int r0, int k0,
                 bool lo = false) {
  const size_t base = img.size();
  img.resize(base + 128 * 128);
  for (int r = 0; r < 128; ++r)
    for (int k = 0; k < 128; ++k) {
      const int byte = (k >> 6) * 128 * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                       ((((k & 63) >> 3) ^ (r & 7)) << 4) + (k & 7) * 2;
      const float v = W[(size_t)(r0 + r) * ld + k0 + k];
      img[base + byte / 2] = to16(v, g_tile_f16, lo);
    }
}

bool build_stream_image(const std::map<std::string, TensorView>& t, bool f16,
                        std::vector<uint16_t>* img) {
  g_tile_f16 = f16;
  auto get = [&](const std::string& n) -> const float* {
    auto it = t.find(n);
    return it == t.end() ? nullptr : it->second.data;
  };
  img->clear();
  for (int l = 0; l < 3; ++l) {
    const std::string p = "decoder_layers." + std::to_string(l) + ".";
    const float* W1 = get(p + "W1.weight");
    const float* W2 = get(p + "W2.weight");
    const float* W3 = get(p + "W3.weight");
    const float* Wi = get(p + "dense.W_in.weight");
    const float* Wo = get(p + "dense.W_out.weight");
    if (!W1 || !W2 || !W3 || !Wi || !Wo) return false;
    if (l > 0) {
      append_tile(*img, W1, 512, 0, 0);     // W1a: h_t block
      append_tile(*img, W1, 512, 0, 384);   // W1d: h_j block
    }
    append_tile(*img, W2, 128, 0, 0);
    append_tile(*img, W3, 128, 0, 0);
    for (int i = 0; i < 4; ++i) {
      append_tile(*img, Wi, 128, 128 * i, 0);         // W_in rows 128i..128i+127
      append_tile(*img, Wi, 128, 128 * i, 0, true);   // and their remainder
    }
    for (int i = 0; i < 4; ++i) append_tile(*img, Wo, 512, 0, 128 * i);   // W_out columns 128i..

  }
  return img->size() == (size_t)kStreamTilesPerStep * 128 * 128;
}

// fp16 GEMM image of rows [r0, r0+nrows) and columns [c0, c0+K) of W
// (row-major, leading dimension ld): [Kp/64 atoms][nrows x 64] SW128.
void append_gemm_image(std::vector<uint16_t>& img, const float* W, int ld, int r0, int nrows,
                       int c0, int K, bool lo = false) {
  const int Kp = (K + 63) & ~63;
  const size_t base = img.size();
  img.resize(base + (size_t)nrows * Kp, 0);
  for (int r = 0; r < nrows; ++r)
    for (int k = 0; k < K; ++k) {
      const size_t byte = (size_t)(k >> 6) * nrows * 128 + (size_t)(r >> 3) * 1024 +
                          (size_t)(r & 7) * 128 + (size_t)((((k & 63) >> 3) ^ (r & 7)) << 4) +
                          (size_t)(k & 7) * 2;
      img[base + byte / 2] = to16(W[(size_t)(r0 + r) * ld + c0 + k], true, lo);
    }
}

// The 16-bit GEMM operands of the fused tensor-core encoder kernels, the
// decoder's slot tables and the node-side GEMMs (gemm_tc3), by name.
bool build_gemm_images(const std::map<std::string, TensorView>& t, std::vector<uint16_t>* img,
                       std::map<std::string, size_t>* at) {
  auto get = [&](const std::string& n) -> const float* {
    auto it = t.find(n);
    return it == t.end() ? nullptr : it->second.data;
  };
  auto mark = [&](const std::string& name) { (*at)[name] = img->size() * 2; };
  const float* We = get("features.edge_embedding.weight");
  const float* WeE = get("W_e.weight");
  if (!We || !WeE) return false;
  mark("edge");
  append_gemm_image(*img, We, 416, 0, 128, 0, 416);
  mark("W_e");
  append_gemm_image(*img, WeE, 128, 0, 128, 0, 128);
  for (int l = 0; l < 3; ++l) {
    const std::string p = "encoder_layers." + std::to_string(l) + ".";
    const std::string q = "enc" + std::to_string(l) + ".";
    // each edge-wise encoder weight also as its remainder image (".lo")
    for (const char* nm : {"W1", "W11"}) {
      const float* W = get(p + nm + ".weight");
      if (!W) return false;
      mark(q + nm + "b");   // the h_E input block
      append_gemm_image(*img, W, 384, 0, 128, 128, 128);
      mark(q + nm + "b.lo");
      append_gemm_image(*img, W, 384, 0, 128, 128, 128, true);
    }
    for (const char* nm : {"W2", "W12", "W13"}) {
      const float* W = get(p + nm + ".weight");
      if (!W) return false;
      mark(q + nm);
      append_gemm_image(*img, W, 128, 0, 128, 0, 128);
      mark(q + nm + ".lo");
      append_gemm_image(*img, W, 128, 0, 128, 0, 128, true);
    }
  }
  for (int l = 0; l < 3; ++l) {
    const std::string p = "decoder_layers." + std::to_string(l) + ".";
    const std::string q = "dec" + std::to_string(l) + ".";
    const float* W1 = get(p + "W1.weight");
    if (!W1) return false;
    mark(q + "W1b");
    append_gemm_image(*img, W1, 512, 0, 128, 128, 128);
  }
  // Node-side GEMMs (gemm_tc3): value (".hi") and remainder (".lo") images,
  // one 128-row block per 128 output columns, blocks in output order.
  for (int lo = 0; lo < 2; ++lo) {
    const char* sfx = lo ? ".lo" : ".hi";
    for (int l = 0; l < 3; ++l) {
      const std::string p = "encoder_layers." + std::to_string(l) + ".";
      const std::string q = "enc" + std::to_string(l) + ".";
      const float* W1 = get(p + "W1.weight");
      const float* W11 = get(p + "W11.weight");
      const float* W3 = get(p + "W3.weight");
      const float* Wi = get(p + "dense.W_in.weight");
      const float* Wo = get(p + "dense.W_out.weight");
      if (!W1 || !W11 || !W3 || !Wi || !Wo) return false;
      mark(q + "nW1ac" + sfx);   // [W1a | W1c]: the h_i and h_j input blocks
      append_gemm_image(*img, W1, 384, 0, 128, 0, 128, lo);
      append_gemm_image(*img, W1, 384, 0, 128, 256, 128, lo);
      mark(q + "nW11ac" + sfx);
      append_gemm_image(*img, W11, 384, 0, 128, 0, 128, lo);
      append_gemm_image(*img, W11, 384, 0, 128, 256, 128, lo);
      mark(q + "nW3" + sfx);
      append_gemm_image(*img, W3, 128, 0, 128, 0, 128, lo);
      mark(q + "nWin" + sfx);
      for (int nb = 0; nb < 4; ++nb) append_gemm_image(*img, Wi, 128, 128 * nb, 128, 0, 128, lo);
      mark(q + "nWout" + sfx);
      append_gemm_image(*img, Wo, 512, 0, 128, 0, 512, lo);
    }
    for (int l = 0; l < 3; ++l) {
      const std::string p = "decoder_layers." + std::to_string(l) + ".";
      const std::string q = "dec" + std::to_string(l) + ".";
      const float* W1 = get(p + "W1.weight");
      mark(q + "nW1d" + sfx);    // the h_j input block
      append_gemm_image(*img, W1, 512, 0, 128, 384, 128, lo);
      if (l == 0) {
        mark(q + "nW1a" + sfx);  // the h_t input block
        append_gemm_image(*img, W1, 512, 0, 128, 0, 128, lo);
      }
    }
  }
  return true;
}

// --------------------------------------------------------------------------
// Batch validation (algorithms/inverse_fold.cpp:232-261 semantics)
// --------------------------------------------------------------------------
bool finite_coords(const float* coords, const uint8_t* src, int64_t R) {
  for (int64_t r = 0; r < R; ++r)
    for (int a = 0; a < 5; ++a) {
      if (!src[r * 5 + a]) continue;
      for (int x = 0; x < 3; ++x)
        if (!std::isfinite(coords[(r * 5 + a) * 3 + x])) return false;
    }
  return true;
}

hkb_status build_host_batch(int B, const int32_t* L, const int32_t* S,
                            const uint8_t* host_src, HostBatch* hb) {
  if (B <= 0) return invalid("batch must contain at least one protein");
  if (L == nullptr || S == nullptr) return invalid("residue_counts and num_seqs must be non-null");
  hb->B = B;
  hb->L.assign(L, L + B);
  hb->S.assign(S, S + B);
  hb->off.resize(B);
  hb->qoff.resize(B);
  hb->seq_base.resize(B);
  int64_t R = 0, Q = 0;
  int64_t NS = 0;
  int max_len = 0;
  for (int b = 0; b < B; ++b) {
    if (L[b] <= 0) return invalid("inverse-fold structure must contain at least one residue");
    if (L[b] > kMaxResidues) return invalid("protein longer than the engine limit of 4096 residues");
    if (S[b] <= 0) return invalid("inverse-fold num_seqs must be greater than zero");
    hb->off[b] = (int)R;
    hb->qoff[b] = Q;
    hb->seq_base[b] = (int)NS;
    R += L[b];
    Q += (int64_t)S[b] * L[b];
    NS += S[b];
    max_len = std::max(max_len, (int)L[b]);
  }
  if (R > (int64_t)1 << 30 || NS > (int64_t)1 << 30) return invalid("batch too large");
  hb->R = (int)R;
  hb->Q = Q;
  hb->NS = (int)NS;
  hb->max_len = max_len;
  hb->res_prot.resize(R);
  hb->seq_prot.resize(NS);
  hb->seq_row_off.resize(NS);
  for (int b = 0; b < B; ++b) {
    for (int i = 0; i < L[b]; ++i) hb->res_prot[hb->off[b] + i] = b;
    for (int s = 0; s < S[b]; ++s) {
      hb->seq_prot[hb->seq_base[b] + s] = b;
      hb->seq_row_off[hb->seq_base[b] + s] = hb->qoff[b] + (int64_t)s * L[b];
    }
  }
  hb->mask.resize(R);
  for (int64_t r = 0; r < R; ++r) {
    const uint8_t* s = host_src + r * 5;
    hb->mask[r] = (s[0] && s[1] && s[2] && s[3]) ? 1.0f : 0.0f;
  }
  return kOk;
}

// Decoding orders for every sequence, on host threads.
// Order-mode and input-permutation checks (decode_order_scalar.cpp:68-82),
// done before any device work is queued.
hkb_status validate_orders(const int32_t* modes, const int32_t* input_orders,
                           const HostBatch& hb) {
  for (int b = 0; b < hb.B; ++b) {
    const int mode = modes ? modes[b] : HKB_DECODE_RANDOM;
    if (mode == HKB_DECODE_INPUT) {
      if (input_orders == nullptr)
        return invalid("ProteinMPNN input decoding_order must be a permutation");
      if (!check_permutation(input_orders + hb.off[b], hb.L[b]))
        return invalid("ProteinMPNN input decoding_order must be a permutation");
    } else if (mode != HKB_DECODE_RANDOM && mode != HKB_DECODE_N_TO_C) {
      return invalid("unknown decode order mode");
    }
  }
  return kOk;
}

// Cores this process may run on (its affinity mask), not the machine's: one
// process per GPU on a shared host each gets its own slice.
int usable_cores() {
  cpu_set_t set;
  CPU_ZERO(&set);
  if (sched_getaffinity(0, sizeof(set), &set) == 0) return std::max(1, CPU_COUNT(&set));
  return (int)std::max(1u, std::thread::hardware_concurrency());
}

// Per-sequence decoding orders of a validated batch (host threads).
void generate_orders(const int32_t* modes, const int32_t* input_orders, HostBatch* hb) {
  hb->orders.assign(hb->Q, 0);
  const int NS = hb->NS;
  auto work = [&](int lo, int hi) {
    for (int sq = lo; sq < hi; ++sq) {
      const int b = hb->seq_prot[sq];
      const int L = hb->L[b];
      int32_t* o = hb->orders.data() + hb->seq_row_off[sq];
      const int mode = modes ? modes[b] : HKB_DECODE_RANDOM;
      if (mode == HKB_DECODE_RANDOM) {
        random_decode_order(hb->mask.data() + hb->off[b], L, hb->seq_seed[sq], o);
      } else if (mode == HKB_DECODE_N_TO_C) {
        for (int p = 0; p < L; ++p) o[p] = p;
      } else {
        std::memcpy(o, input_orders + hb->off[b], sizeof(int32_t) * L);
      }
    }
  };
  const int64_t work_items = hb->Q;
  int nthreads = (int)std::min<int64_t>(usable_cores(), std::max<int64_t>(1, work_items / 16384));
  nthreads = std::min(nthreads, 32);
  if (nthreads <= 1 || NS < 2) {
    work(0, NS);
  } else {
    std::vector<std::thread> th;
    const int per = (NS + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; ++t) {
      const int lo = t * per, hi = std::min(NS, lo + per);
      if (lo >= hi) break;
      th.emplace_back(work, lo, hi);
    }
    for (auto& x : th) x.join();
  }
}

hkb_status build_orders(const int32_t* modes, const int32_t* input_orders, HostBatch* hb) {
  hkb_status s = validate_orders(modes, input_orders, *hb);
  if (s.code != HKB_OK) return s;
  generate_orders(modes, input_orders, hb);
  return kOk;
}

// Uploads the per-batch tables; returns the BatchView.
hkb_status upload_tables(hkb_engine* e, const HostBatch& hb, DeviceBatch* db) {
  auto& ws = e->ws;
  int* prot_off = ws.get_as<int>("t.prot_off", hb.B);
  int* prot_len = ws.get_as<int>("t.prot_len", hb.B);
  int* res_prot = ws.get_as<int>("t.res_prot", hb.R);
  int* seq_prot = ws.get_as<int>("t.seq_prot", hb.NS);
  int64_t* seq_row = ws.get_as<int64_t>("t.seq_row", hb.NS);
  if (!prot_off || !prot_len || !res_prot || !seq_prot || !seq_row)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  cudaStream_t st = e->stream;
  HKB_CUDA(cudaMemcpyAsync(prot_off, hb.off.data(), sizeof(int) * hb.B, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(prot_len, hb.L.data(), sizeof(int) * hb.B, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(res_prot, hb.res_prot.data(), sizeof(int) * hb.R, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(seq_prot, hb.seq_prot.data(), sizeof(int) * hb.NS, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(seq_row, hb.seq_row_off.data(), sizeof(int64_t) * hb.NS, cudaMemcpyHostToDevice, st));
  BatchView& bv = db->bv;
  bv.num_proteins = hb.B;
  bv.total_residues = hb.R;
  bv.total_rows = hb.Q;
  bv.num_sequences = hb.NS;
  bv.prot_res_off = prot_off;
  bv.prot_len = prot_len;
  bv.res_prot = res_prot;
  bv.seq_prot = seq_prot;
  bv.seq_row_off = seq_row;
  return kOk;
}

// --------------------------------------------------------------------------
// Device pipeline (fp32)
// --------------------------------------------------------------------------
hkb_status encode_f32(hkb_engine* e, const HostBatch& hb, const DeviceBatch& db,
                      EncoderOut* eo) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const F32Weights& w = e->w32;
  const int64_t R = hb.R, SL = R * kK;
  eo->e_idx = ws.get_as<int>("e.idx", SL);
  eo->d2 = ws.get_as<float>("e.d2", SL);
  eo->mask = ws.get_as<float>("e.mask", R);
  eo->h_e = ws.get_as<float>("e.he", SL * kH);
  eo->h_v = ws.get_as<float>("e.hv", R * kH);
  float* feat = ws.get_as<float>("e.feat", SL * kEdgeIn);
  float* E1 = ws.get_as<float>("e.s1", SL * kH);
  float* EB = ws.get_as<float>("e.s2", SL * kH);
  float* G1 = ws.get_as<float>("e.s3", SL * kH);
  float* NAC = ws.get_as<float>("e.nac", R * 256);
  float* Sv = ws.get_as<float>("e.S", R * kH);
  float* cnt = ws.get_as<float>("e.cnt", R);
  float* T3 = ws.get_as<float>("e.T3", R * kH);
  float* h1 = ws.get_as<float>("e.h1", R * kH);
  float* F = ws.get_as<float>("e.F", R * kFfn);
  float* Y = ws.get_as<float>("e.Y", R * kH);
  if (!eo->e_idx || !eo->d2 || !eo->mask || !eo->h_e || !eo->h_v || !feat || !E1 ||
      !EB || !G1 || !NAC || !Sv || !cnt || !T3 || !h1 || !F || !Y)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  const BatchView& bv = db.bv;
  int64_t& n = e->launches;
  launch_knn(st, bv, db.coords, db.sources, eo->e_idx, eo->d2, eo->mask, e->d_err, hb.max_len);
  launch_edge_features(st, bv, w, db.coords, db.sources, eo->e_idx, feat);
  gemm_f32(st, SL, kH, kEdgeIn, feat, kEdgeIn, w.edge_wT, kH, nullptr, 0, E1, kH);
  launch_ln_rows(st, SL, E1, nullptr, nullptr, w.norm_e_w, w.norm_e_b, nullptr, nullptr, E1);
  gemm_f32(st, SL, kH, kH, E1, kH, w.We_T, kH, w.We_b, 0, eo->h_e, kH);
  HKB_CUDA(cudaMemsetAsync(eo->h_v, 0, sizeof(float) * R * kH, st));
  n += 5;
  for (int l = 0; l < 3; ++l) {
    const auto& E = w.enc[l];
    gemm_f32(st, R, 256, kH, eo->h_v, kH, E.W1acT, 256, E.b1ac, 0, NAC, 256);
    gemm_f32(st, SL, kH, kH, eo->h_e, kH, E.W1bT, kH, nullptr, 0, EB, kH);
    launch_enc_msg_in(st, bv, NAC, EB, eo->e_idx, G1);
    gemm_f32(st, SL, kH, kH, G1, kH, E.W2T, kH, E.b2, 1, EB, kH);
    launch_enc_aggregate(st, bv, EB, eo->e_idx, eo->mask, Sv, cnt);
    gemm_f32(st, R, kH, kH, Sv, kH, E.W3T, kH, nullptr, 0, T3, kH);
    launch_enc_node_update(st, bv, T3, cnt, E.b3, eo->h_v, E.n1w, E.n1b, h1);
    gemm_f32(st, R, kFfn, kH, h1, kH, E.WinT, kFfn, E.bin, 1, F, kFfn);
    gemm_f32(st, R, kH, kFfn, F, kFfn, E.WoutT, kH, nullptr, 0, Y, kH);
    launch_ln_rows(st, R, h1, Y, E.bout, E.n2w, E.n2b, eo->mask, nullptr, eo->h_v);
    gemm_f32(st, R, 256, kH, eo->h_v, kH, E.W11acT, 256, E.b11ac, 0, NAC, 256);
    gemm_f32(st, SL, kH, kH, eo->h_e, kH, E.W11bT, kH, nullptr, 0, EB, kH);
    launch_enc_msg_in(st, bv, NAC, EB, eo->e_idx, G1);
    gemm_f32(st, SL, kH, kH, G1, kH, E.W12T, kH, E.b12, 1, EB, kH);
    gemm_f32(st, SL, kH, kH, EB, kH, E.W13T, kH, E.b13, 0, G1, kH);
    launch_edge_ln_update(st, bv, G1, eo->e_idx, E.n3w, E.n3b, eo->h_e);
    n += 16;
  }
  HKB_CUDA(cudaGetLastError());
  return kOk;
}

hkb_status decoder_tables_f32(hkb_engine* e, const HostBatch& hb, const EncoderOut& eo,
                              DecoderTables* dt) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const F32Weights& w = e->w32;
  const int64_t R = hb.R, SL = R * kK;
  for (int l = 0; l < 3; ++l) {
    float* pe = ws.get_as<float>("d.PE" + std::to_string(l), SL * kH);
    float* pv = ws.get_as<float>("d.PVenc" + std::to_string(l), R * kH);
    if (!pe || !pv) return {HKB_UNAVAILABLE, "device allocation failed"};
    gemm_f32(st, SL, kH, kH, eo.h_e, kH, w.dec[l].W1bT, kH, nullptr, 0, pe, kH);
    gemm_f32(st, R, kH, kH, eo.h_v, kH, w.dec[l].W1dT, kH, nullptr, 0, pv, kH);
    dt->PE[l] = pe;
    dt->PVenc[l] = pv;
  }
  float* a0 = ws.get_as<float>("d.Aenc0", R * kH);
  if (!a0) return {HKB_UNAVAILABLE, "device allocation failed"};
  gemm_f32(st, R, kH, kH, eo.h_v, kH, w.dec[0].W1aT, kH, w.dec[0].b1, 0, a0, kH);
  dt->Aenc0 = a0;
  e->launches += 7;
  return kOk;
}

// Tensor-core encoder: the same pipeline as encode_f32 with every slot-sized
// and node-sized contraction on tcgen05 (fp16 operands, fp32 accumulation,
// fp32 intermediates); gathers, aggregation and LayerNorms stay as they are.
hkb_status encode_tc(hkb_engine* e, const HostBatch& hb, const DeviceBatch& db,
                     EncoderOut* eo) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const F32Weights& w = e->w32;
  const int64_t R = hb.R, SL = R * kK;
  eo->e_idx = ws.get_as<int>("e.idx", SL);
  eo->d2 = ws.get_as<float>("e.d2", SL);
  eo->mask = ws.get_as<float>("e.mask", R);
  eo->h_e = nullptr;
  // h_E (value) holds at least one TMA box of rows (kNodeTileRows), so the
  // tensor maps of the encoder passes never describe fewer rows than a box;
  // rows past SL are zero
  eo->h_e_rows = SL < kNodeTileRows ? (int64_t)kNodeTileRows : SL;
  eo->h_e16 = ws.get_as<uint16_t>("e.he16", eo->h_e_rows * kH);
  eo->h_e16lo = ws.get_as<uint16_t>("e.he16lo", SL * kH);
  eo->h_v = ws.get_as<float>("e.hv", R * kH);
  float* NAC = ws.get_as<float>("e.nac", R * 256);
  float* Sv = ws.get_as<float>("e.S", R * kH);
  float* cnt = ws.get_as<float>("e.cnt", R);
  float* T3 = ws.get_as<float>("e.T3", R * kH);
  float* h1 = ws.get_as<float>("e.h1", R * kH);
  float* F = ws.get_as<float>("e.F", R * kFfn);
  float* Y = ws.get_as<float>("e.Y", R * kH);
  if (!eo->e_idx || !eo->d2 || !eo->mask || !eo->h_e16 || !eo->h_e16lo || !eo->h_v || !NAC || !Sv || !cnt ||
      !T3 || !h1 || !F || !Y)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  const BatchView& bv = db.bv;
  // Node-side GEMMs (M = R residue rows) on tcgen05 with both operands as
  // fp16 value + remainder (about 22 significant bits each, close to fp32:
  // their 16-bit rounding would be the largest error source of the encoder).
  auto lin = [&](int N, int K, const float* A, int lda, const std::string& W, const float* bias,
                 int act, float* C, int ldc) {
    gemm_tc3(st, R, N, K, A, lda, e->gemm_img.at(W + ".hi"), e->gemm_img.at(W + ".lo"), bias,
             act, C, ldc, false, e->d_err);
    e->launches += 1;
  };
  launch_knn(st, bv, db.coords, db.sources, eo->e_idx, eo->d2, eo->mask, e->d_err, hb.max_len);
  EncFeatTcArgs fa;
  fa.bv = bv;
  fa.coords = db.coords;
  fa.src = db.sources;
  fa.e_idx = eo->e_idx;
  fa.pos_w = w.pos_w;
  fa.pos_b = w.pos_b;
  fa.Wedge = e->gemm_img.at("edge");
  fa.We = e->gemm_img.at("W_e");
  fa.ln_w = w.norm_e_w;
  fa.ln_b = w.norm_e_b;
  fa.We_b = w.We_b;
  fa.h_e = eo->h_e16;
  fa.h_e_lo = eo->h_e16lo;
  fa.err = e->d_err;
  launch_enc_featurize_tc(st, fa, e->num_sms);
  e->launches += 2;   // kNN, featurisation (memsets are not counted)
  HKB_CUDA(cudaMemsetAsync(eo->h_v, 0, sizeof(float) * R * kH, st));
  // TMA tensor maps of h_E (value) for the node and edge passes' tile loads
  if (eo->h_e_rows > SL)
    HKB_CUDA(cudaMemsetAsync(eo->h_e16 + SL * kH, 0,
                             sizeof(uint16_t) * (size_t)(eo->h_e_rows - SL) * kH, st));
  CUtensorMap map_node, map_edge;
  if (!make_rows_tensor_map(&map_node, eo->h_e16, eo->h_e_rows, kNodeTileRows) ||
      !make_rows_tensor_map(&map_edge, eo->h_e16, eo->h_e_rows, 128))
    return internal("TMA tensor map encoding failed");
  for (int l = 0; l < 3; ++l) {
    const auto& E = w.enc[l];
    const std::string q = "enc" + std::to_string(l) + ".";
    // node messages: one fused pass over h_E (W1b, gathers, GELU, W2, GELU, slot sum)
    lin(256, kH, eo->h_v, kH, q + "nW1ac", E.b1ac, 0, NAC, 256);
    EncNodeTcArgs na;
    na.map_he = map_node;
    na.bv = bv;
    na.h_e = eo->h_e16;
    na.e_idx = eo->e_idx;
    na.mask = eo->mask;
    na.NAC = NAC;
    na.W1b = e->gemm_img.at(q + "W1b");
    na.W2 = e->gemm_img.at(q + "W2");
    na.W1b_lo = e->gemm_img.at(q + "W1b.lo");
    na.W2_lo = e->gemm_img.at(q + "W2.lo");
    na.b2 = E.b2;
    na.S = Sv;
    na.cnt = cnt;
    na.err = e->d_err;
    launch_enc_node_tc(st, na, e->num_sms);
    lin(kH, kH, Sv, kH, q + "nW3", nullptr, 0, T3, kH);
    launch_enc_node_update(st, bv, T3, cnt, E.b3, eo->h_v, E.n1w, E.n1b, h1);
    lin(kFfn, kH, h1, kH, q + "nWin", E.bin, 1, F, kFfn);
    lin(kH, kFfn, F, kFfn, q + "nWout", nullptr, 0, Y, kH);
    launch_ln_rows(st, R, h1, Y, E.bout, E.n2w, E.n2b, eo->mask, nullptr, eo->h_v);
    // edge update: one fused pass (W11b, gathers, GELU, W12, GELU, W13, LN3)
    lin(256, kH, eo->h_v, kH, q + "nW11ac", E.b11ac, 0, NAC, 256);
    EncEdgeTcArgs ea;
    ea.map_he = map_edge;
    ea.bv = bv;
    ea.h_e = eo->h_e16;
    ea.h_e_out = eo->h_e16;
    ea.h_e_lo = eo->h_e16lo;
    ea.e_idx = eo->e_idx;
    ea.NAC = NAC;
    ea.W11b = e->gemm_img.at(q + "W11b");
    ea.W12 = e->gemm_img.at(q + "W12");
    ea.W13 = e->gemm_img.at(q + "W13");
    ea.W11b_lo = e->gemm_img.at(q + "W11b.lo");
    ea.W12_lo = e->gemm_img.at(q + "W12.lo");
    ea.W13_lo = e->gemm_img.at(q + "W13.lo");
    ea.b12 = E.b12;
    ea.b13 = E.b13;
    ea.n3w = E.n3w;
    ea.n3b = E.n3b;
    ea.err = e->d_err;
    launch_enc_edge_tc(st, ea, e->num_sms);
    e->launches += 4;
  }
  HKB_CUDA(cudaGetLastError());
  return kOk;
}

// Decoder tables straight to 16-bit (fp16 mode) for the fused decode kernel.
hkb_status decoder_tables_tc(hkb_engine* e, const HostBatch& hb, const BatchView& db_bv,
                             const EncoderOut& eo, Bf16DecodeTables* tb, bool with_pe = true) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const int64_t R = hb.R, SL = R * kK;
  DecTablesTcArgs ta;
  if (with_pe && !make_rows_tensor_map(&ta.map_he, eo.h_e16, eo.h_e_rows, 128))
    return internal("TMA tensor map encoding failed");
  ta.bv = db_bv;
  ta.e_idx = eo.e_idx;
  ta.h_e = eo.h_e16;
  ta.rows = SL;
  ta.err = e->d_err;
  for (int l = 0; l < 3; ++l) {
    uint16_t* pe = with_pe ? ws.get_as<uint16_t>("b.PE" + std::to_string(l), SL * kH) : nullptr;
    uint16_t* pv = ws.get_as<uint16_t>("b.PVenc" + std::to_string(l), R * kH);
    if ((with_pe && !pe) || !pv) return {HKB_UNAVAILABLE, "device allocation failed"};
    const std::string q = "dec" + std::to_string(l) + ".";
    ta.W[l] = e->gemm_img.at(q + "W1b");
    ta.PVenc[l] = pv;
    ta.out[l] = pe;
    // W1d h_enc per residue (value + remainder products, about fp32
    // precision) rounded once to the 16-bit table
    gemm_tc3(st, R, kH, kH, eo.h_v, kH, e->gemm_img.at(q + "nW1d.hi"),
             e->gemm_img.at(q + "nW1d.lo"), nullptr, 0, pv, kH, true, e->d_err);
    tb->PE[l] = pe;
    tb->PVenc[l] = pv;
  }
  // (the teacher-forced pass forms W1b h_E by MMA from h_E itself)
  if (with_pe) launch_dec_tables_tc(st, ta, e->num_sms);
  float* a0 = ws.get_as<float>("d.Aenc0", R * kH);
  if (!a0) return {HKB_UNAVAILABLE, "device allocation failed"};
  gemm_tc3(st, R, kH, kH, eo.h_v, kH, e->gemm_img.at("dec0.nW1a.hi"),
           e->gemm_img.at("dec0.nW1a.lo"), e->w32.dec[0].b1, 0, a0, kH, false, e->d_err);
  tb->Aenc0 = a0;
  tb->h_enc = eo.h_v;
  e->launches += with_pe ? 5 : 4;   // 3 PVenc GEMMs, [slot tables,] Aenc0
  HKB_CUDA(cudaGetLastError());
  return kOk;
}

struct DeviceDesignOut {
  int* tokens;
  float* log_probs;
  int* orders;
  float* scores;
};

hkb_status decode_f32(hkb_engine* e, const HostBatch& hb, const DeviceBatch& db,
                      const EncoderOut& eo, const DecoderTables& dt,
                      const DeviceDesignOut& o) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const int G = ar_f32_group_size();
  std::vector<int> g0, gc;
  for (int b = 0; b < hb.B; ++b)
    for (int s = 0; s < hb.S[b]; s += G) {
      g0.push_back(hb.seq_base[b] + s);
      gc.push_back(std::min(G, hb.S[b] - s));
    }
  const int ng = (int)g0.size();
  int* d_g0 = ws.get_as<int>("a.g0", ng);
  int* d_gc = ws.get_as<int>("a.gc", ng);
  int* pos = ws.get_as<int>("a.pos", hb.Q);
  float* PV = ws.get_as<float>("a.PV", 2 * hb.Q * kH);
  uint64_t* seeds = ws.get_as<uint64_t>("a.seed", hb.NS);
  float* temps = ws.get_as<float>("a.temp", hb.NS);
  if (!d_g0 || !d_gc || !pos || !PV || !seeds || !temps)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_g0, g0.data(), sizeof(int) * ng, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_gc, gc.data(), sizeof(int) * ng, cudaMemcpyHostToDevice, st));
  // seeds and temperatures were uploaded with the decoding orders
  HKB_CUDA(cudaMemsetAsync(PV, 0, sizeof(float) * 2 * hb.Q * kH, st));
  ArArgs a{};
  a.group_seq0 = d_g0;
  a.group_count = d_gc;
  a.num_groups = ng;
  a.orders = o.orders;
  a.pos = pos;
  a.tokens = o.tokens;
  a.log_probs = o.log_probs;
  a.scores = o.scores;
  a.PV = PV;
  a.seq_seed = seeds;
  a.seq_temp = temps;
  a.mask = eo.mask;
  a.e_idx = eo.e_idx;
  a.h_enc = eo.h_v;
  a.total_rows = hb.Q;
  launch_ar_decode_f32(st, db.bv, e->w32, dt, a, e->d_err);
  launch_scores(st, db.bv, o.tokens, o.log_probs, eo.mask, o.scores);
  e->launches += 2;
  (void)db;
  return kOk;
}

// bf16 mode: the fp32 decoder tables rounded to bf16.
hkb_status decoder_tables_bf16(hkb_engine* e, const HostBatch& hb, const BatchView& db_bv,
                               const EncoderOut& eo, const DecoderTables& dt,
                               Bf16DecodeTables* tb) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const int64_t R = hb.R, SL = R * kK;
  for (int l = 0; l < 3; ++l) {
    uint16_t* pe = ws.get_as<uint16_t>("b.PE" + std::to_string(l), SL * kH);
    uint16_t* pv = ws.get_as<uint16_t>("b.PVenc" + std::to_string(l), R * kH);
    if (!pe || !pv) return {HKB_UNAVAILABLE, "device allocation failed"};
    convert_f32_to_16(st, dt.PVenc[l], pv, R * kH, false);
    presum_slot_table(st, db_bv, eo.e_idx, dt.PE[l], pv, pe, false);
    tb->PE[l] = pe;
    tb->PVenc[l] = pv;
  }
  tb->Aenc0 = dt.Aenc0;
  tb->h_enc = eo.h_v;
  e->launches += 6;
  return kOk;
}

// Sequence groups of the fused decode kernel (one CTA each).  A group holds
// sequences of proteins with the same length (the CTA walks L positions);
// groups are listed longest protein first, and each length bucket is split
// into near-equal groups of at most ceil(NS / SMs) sequences (capped at
// `max_group`), so that a batch that fits one wave of CTAs fills every SM.
// `seqs` is [groups, max_group], padded with -1.
void build_decode_groups(const HostBatch& hb, int max_group, int num_sms,
                         std::vector<int>* seqs, std::vector<int>* counts) {
  std::map<int, std::vector<int>, std::greater<int>> by_len;
  for (int sq = 0; sq < hb.NS; ++sq) by_len[hb.L[hb.seq_prot[sq]]].push_back(sq);
  const int G = std::min(max_group, std::max(1, (hb.NS + num_sms - 1) / std::max(1, num_sms)));
  seqs->clear();
  counts->clear();
  for (const auto& kv : by_len) {
    const std::vector<int>& list = kv.second;
    const int n = (int)list.size();
    const int ng = (n + G - 1) / G;
    const int base = n / ng, extra = n % ng;
    int at = 0;
    for (int g = 0; g < ng; ++g) {
      const int c = base + (g < extra ? 1 : 0);
      counts->push_back(c);
      for (int i = 0; i < max_group; ++i) seqs->push_back(i < c ? list[at + i] : -1);
      at += c;
    }
  }
}

hkb_status decode_tc(hkb_engine* e, const HostBatch& hb, const DeviceBatch& db,
                     const EncoderOut& eo, const Bf16DecodeTables& tb,
                     const DeviceDesignOut& o) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const bool f16 = e->precision == HKB_PRECISION_F16;
  const int G = ar_tc_group_size();
  std::vector<int> gseq, gc;
  build_decode_groups(hb, G, e->num_sms, &gseq, &gc);
  const int ng = (int)gc.size();
  int* d_g0 = ws.get_as<int>("a.gseq", (size_t)ng * G);
  int* d_gc = ws.get_as<int>("a.gc", ng);
  int* pos = ws.get_as<int>("a.pos", hb.Q);
  float* lp_tok = ws.get_as<float>("a.lptok", hb.Q);
  uint16_t* PV = ws.get_as<uint16_t>("b.PV", 2 * hb.Q * kH);
  uint64_t* seeds = ws.get_as<uint64_t>("a.seed", hb.NS);
  float* temps = ws.get_as<float>("a.temp", hb.NS);
  if (!d_g0 || !d_gc || !pos || !lp_tok || !PV || !seeds || !temps)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_g0, gseq.data(), sizeof(int) * gseq.size(), cudaMemcpyHostToDevice,
                           st));
  HKB_CUDA(cudaMemcpyAsync(d_gc, gc.data(), sizeof(int) * ng, cudaMemcpyHostToDevice, st));
  // seeds and temperatures were uploaded with the decoding orders
  ArBf16Args a{};
  a.group_seqs = d_g0;
  a.group_count = d_gc;
  a.num_groups = ng;
  a.orders = o.orders;
  a.pos = pos;
  a.tokens = o.tokens;
  a.log_probs = o.log_probs;
  a.lp_tok = lp_tok;
  a.PV = PV;
  a.seq_seed = seeds;
  a.seq_temp = temps;
  a.mask = eo.mask;
  a.e_idx = eo.e_idx;
  a.total_rows = hb.Q;
  if (e->stall_check_calls > 0) {
    a.stall_check = 1;
    --e->stall_check_calls;
  }
  launch_ar_decode_tc(st, db.bv, e->wbf, tb, a, f16, e->d_err);
  // the scores read the sampled tokens' log-probs from lp_tok, never the
  // [Q,21] rows, which may live in mapped host memory
  launch_scores(st, db.bv, o.tokens, o.log_probs, eo.mask, o.scores, lp_tok);
  e->launches += 2;
  return kOk;
}

hkb_status check_device_error(hkb_engine* e) {
  unsigned int h = 0;
  HKB_CUDA(cudaMemcpyAsync(&h, e->d_err, sizeof(unsigned int), cudaMemcpyDeviceToHost,
                           e->stream));
  HKB_CUDA(cudaStreamSynchronize(e->stream));
  if (h & kErrTimeout) return internal("device wait timed out");
  if (h & kErrTmemAlloc) return internal("tensor-memory allocation failed");
  if (h & kErrBadIndex) return internal("device kernel saw an out-of-range index");
  return kOk;
}


// Pinned staging for host-recomputed orders, `rows` entries; waits for the
// previous upload out of it first.
hkb_status order_staging(hkb_engine* e, int64_t rows, int32_t** out) {
  if (e->h_orders_cap < (size_t)rows) {
    if (e->h_orders) {
      HKB_CUDA(cudaEventSynchronize(e->ev_orders));
      cudaFreeHost(e->h_orders);
      e->h_orders = nullptr;
      e->h_orders_cap = 0;
    }
    if (cudaMallocHost(&e->h_orders, sizeof(int32_t) * rows) != cudaSuccess) {
      cudaGetLastError();
      e->h_orders = nullptr;
      return {HKB_UNAVAILABLE, "host allocation failed"};
    }
    e->h_orders_cap = rows;
  } else {
    HKB_CUDA(cudaEventSynchronize(e->ev_orders));
  }
  *out = e->h_orders;
  return kOk;
}

// Queues the device decoding-order kernel into `orders` [Q] and the read-back
// of the list of sequences the host must recompute.
hkb_status launch_orders(hkb_engine* e, const HostBatch& hb, const int32_t* modes_in,
                         const int32_t* input_orders, const DeviceBatch& db, int32_t* orders) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  uint64_t* seeds = ws.get_as<uint64_t>("a.seed", hb.NS);
  float* temps = ws.get_as<float>("a.temp", hb.NS);
  int* modes = ws.get_as<int>("o.modes", hb.B);
  unsigned int* rc = ws.get_as<unsigned int>("o.recheck", 1 + kRecheckCap);
  if (!seeds || !temps || !modes || !rc) return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(seeds, hb.seq_seed.data(), sizeof(uint64_t) * hb.NS,
                           cudaMemcpyHostToDevice, st));
  if (hb.seq_temp.size() == (size_t)hb.NS)
    HKB_CUDA(cudaMemcpyAsync(temps, hb.seq_temp.data(), sizeof(float) * hb.NS,
                             cudaMemcpyHostToDevice, st));
  std::vector<int> m(hb.B);
  bool any_input = false;
  for (int b = 0; b < hb.B; ++b) {
    m[b] = modes_in ? modes_in[b] : HKB_DECODE_RANDOM;
    any_input |= m[b] == HKB_DECODE_INPUT;
  }
  HKB_CUDA(cudaMemcpyAsync(modes, m.data(), sizeof(int) * hb.B, cudaMemcpyHostToDevice, st));
  OrderArgs oa;
  oa.bv = db.bv;
  oa.sources = db.sources;
  oa.modes = modes;
  if (any_input) {
    int32_t* io = ws.get_as<int32_t>("o.input", hb.R);
    if (!io) return {HKB_UNAVAILABLE, "device allocation failed"};
    HKB_CUDA(cudaMemcpyAsync(io, input_orders, sizeof(int32_t) * hb.R,
                             cudaMemcpyHostToDevice, st));
    HKB_CUDA(cudaStreamSynchronize(st));   // pageable source: copy before returning
    oa.input_orders = io;
  }
  oa.seeds = seeds;
  oa.orders = orders;
  oa.recheck_count = rc;
  oa.recheck_list = reinterpret_cast<int*>(rc + 1);
  oa.recheck_cap = kRecheckCap;
  oa.recheck_all = e->recheck_all_orders;
  oa.err = e->d_err;
  HKB_CUDA(cudaMemsetAsync(rc, 0, sizeof(unsigned int), st));
  launch_decode_orders(st, oa);
  e->launches += 1;
  HKB_CUDA(cudaMemcpyAsync(e->h_recheck, rc, sizeof(unsigned int) * (1 + kRecheckCap),
                           cudaMemcpyDeviceToHost, st));
  HKB_CUDA(cudaEventRecord(e->ev_recheck, st));
  return kOk;
}

// Waits for the order kernel's recheck list and recomputes the listed
// sequences' random orders with the host libm (the reference's arithmetic),
// uploading them over the device's before the decode reads them.
hkb_status finish_orders(hkb_engine* e, HostBatch& hb, const int32_t* modes_in,
                         int32_t* orders) {
  HKB_CUDA(cudaEventSynchronize(e->ev_recheck));
  const unsigned int n = e->h_recheck[0];
  if (n == 0) return kOk;
  std::vector<int> list;
  if (n <= (unsigned int)kRecheckCap) {
    list.assign(reinterpret_cast<const int*>(e->h_recheck + 1),
                reinterpret_cast<const int*>(e->h_recheck + 1) + n);
    std::sort(list.begin(), list.end());
  } else {
    for (int sq = 0; sq < hb.NS; ++sq) {
      const int mode = modes_in ? modes_in[hb.seq_prot[sq]] : HKB_DECODE_RANDOM;
      if (mode == HKB_DECODE_RANDOM) list.push_back(sq);
    }
  }
  int64_t rows = 0;
  for (int sq : list) rows += hb.L[hb.seq_prot[sq]];
  int32_t* stage = nullptr;
  hkb_status s = order_staging(e, rows, &stage);
  if (s.code != HKB_OK) return s;
  int64_t at = 0;
  for (int sq : list) {
    const int b = hb.seq_prot[sq];
    random_decode_order(hb.mask.data() + hb.off[b], hb.L[b], hb.seq_seed[sq], stage + at);
    HKB_CUDA(cudaMemcpyAsync(orders + hb.seq_row_off[sq], stage + at, sizeof(int32_t) * hb.L[b],
                             cudaMemcpyHostToDevice, e->stream));
    at += hb.L[b];
  }
  HKB_CUDA(cudaEventRecord(e->ev_orders, e->stream));
  e->orders_rechecked += (int64_t)list.size();
  return kOk;
}

hkb_status design_common(hkb_engine* e, const hkb_design_batch* batch,
                         const uint8_t* host_src, const float* d_coords,
                         const uint8_t* d_src, HostBatch* hb,
                         const DeviceDesignOut& out) {
  for (int b = 0; b < batch->num_proteins; ++b) {
    const float T = batch->temperatures ? batch->temperatures[b] : 0.1f;
    if (!std::isfinite(T) || T < 0.0f)
      return invalid("inverse-fold sampling_temp must be finite and >= 0");
  }
  hkb_status s = build_host_batch(batch->num_proteins, batch->residue_counts,
                                  batch->num_seqs, host_src, hb);
  if (s.code != HKB_OK) return s;
  hb->seq_seed.resize(hb->NS);
  hb->seq_temp.resize(hb->NS);
  for (int b = 0; b < hb->B; ++b)
    for (int q = 0; q < hb->S[b]; ++q) {
      const int sq = hb->seq_base[b] + q;
      hb->seq_seed[sq] = (batch->seeds ? batch->seeds[b] : 0ull) + (uint64_t)q;
      hb->seq_temp[sq] = batch->temperatures ? batch->temperatures[b] : 0.1f;
    }
  s = validate_orders(batch->decode_orders, batch->input_orders, *hb);
  if (s.code != HKB_OK) return s;
  e->launches = 0;
  cudaStream_t st = e->stream;
  HKB_CUDA(cudaMemsetAsync(e->d_err, 0, sizeof(unsigned int), st));
  DeviceBatch db;
  db.coords = d_coords;
  db.sources = d_src;
  s = upload_tables(e, *hb, &db);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[0], st));
  // Decoding orders on the device, ahead of the encoder; the host only
  // recomputes the rare sequences the kernel marks (after the encoder is
  // queued, so the wait overlaps device work).
  s = launch_orders(e, *hb, batch->decode_orders, batch->input_orders, db, out.orders);
  if (s.code != HKB_OK) return s;
  EncoderOut eo;
  // fp32: SIMT parity pipeline; bf16: fp32 encoder, tables rounded to bf16;
  // f16: tensor-core encoder writing fp16 tables.
  const bool tc_encoder = e->precision == HKB_PRECISION_F16;
  {
    PhaseRange r("hkb.featurise+encode");
    s = tc_encoder ? encode_tc(e, *hb, db, &eo) : encode_f32(e, *hb, db, &eo);
  }
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[1], st));
  DecoderTables dt{};
  Bf16DecodeTables tb{};
  {
    PhaseRange r("hkb.decoder_tables");
    if (tc_encoder) {
      s = decoder_tables_tc(e, *hb, db.bv, eo, &tb);
    } else {
      s = decoder_tables_f32(e, *hb, eo, &dt);
      if (s.code == HKB_OK && e->precision == HKB_PRECISION_BF16)
        s = decoder_tables_bf16(e, *hb, db.bv, eo, dt, &tb);
    }
    if (s.code == HKB_OK) s = finish_orders(e, *hb, batch->decode_orders, out.orders);
  }
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[2], st));
  {
    PhaseRange r("hkb.decode");
    s = e->precision == HKB_PRECISION_FP32 ? decode_f32(e, *hb, db, eo, dt, out)
                                            : decode_tc(e, *hb, db, eo, tb, out);
  }
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[3], st));
  HKB_CUDA(cudaGetLastError());
  return kOk;
}

void record_timings(hkb_engine* e);

// Teacher-forced scoring of an fp16 engine on tensor cores: the tensor-core
// encoder, the per-residue decoder tables, then per decoder layer one slot
// pass and one node pass over all (sequence, residue) rows.  `hb` holds the
// validated batch; device inputs are uploaded here.
hkb_status score_tc(hkb_engine* e, const hkb_score_batch* batch, HostBatch& hb,
                    hkb_score_out* out) {
  auto& ws = e->ws;
  cudaStream_t st = e->stream;
  const int64_t Q = hb.Q, R = hb.R;
  e->launches = 0;
  HKB_CUDA(cudaMemsetAsync(e->d_err, 0, sizeof(unsigned int), st));
  float* d_coords = ws.get_as<float>("in.coords", R * 15);
  uint8_t* d_src = ws.get_as<uint8_t>("in.src", R * 5);
  int32_t* d_orders = ws.get_as<int32_t>("o.orders", Q);
  int32_t* d_tok = ws.get_as<int32_t>("tf.tok", Q);
  int* d_pos = ws.get_as<int>("tf.pos", Q);
  int* d_rres = ws.get_as<int>("tf.rres", Q);
  int* d_seq0 = ws.get_as<int>("tf.seq0", hb.B);
  int* d_nseq = ws.get_as<int>("tf.nseq", hb.B);
  float* S = ws.get_as<float>("tf.S", Q * kH);
  float* h = ws.get_as<float>("tf.h", Q * kH);
  float* A = ws.get_as<float>("tf.A", Q * kH);
  uint16_t* PV = ws.get_as<uint16_t>("tf.PV", Q * kH);
  float* LP = ws.get_as<float>("tf.LP", Q * kV);
  float* sc = ws.get_as<float>("tf.sc", hb.NS);
  if (!d_coords || !d_src || !d_orders || !d_tok || !d_pos || !d_rres || !d_seq0 || !d_nseq ||
      !S || !h || !A || !PV || !LP || !sc)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_coords, batch->coords, sizeof(float) * R * 15,
                           cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_src, batch->atom_sources, R * 5, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_tok, batch->tokens, sizeof(int32_t) * Q, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_seq0, hb.seq_base.data(), sizeof(int) * hb.B, cudaMemcpyHostToDevice,
                           st));
  HKB_CUDA(cudaMemcpyAsync(d_nseq, hb.S.data(), sizeof(int) * hb.B, cudaMemcpyHostToDevice, st));
  DeviceBatch db;
  db.coords = d_coords;
  db.sources = d_src;
  hkb_status s = upload_tables(e, hb, &db);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[0], st));
  if (batch->orders) {
    HKB_CUDA(cudaMemcpyAsync(d_orders, batch->orders, sizeof(int32_t) * Q,
                             cudaMemcpyHostToDevice, st));
  } else {
    s = launch_orders(e, hb, nullptr, nullptr, db, d_orders);
    if (s.code != HKB_OK) return s;
  }
  EncoderOut eo;
  {
    PhaseRange r("hkb.featurise+encode");
    s = encode_tc(e, hb, db, &eo);
  }
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[1], st));
  Bf16DecodeTables tb{};
  PhaseRange r_tab("hkb.decoder_tables+teacher_forced_layers");
  s = decoder_tables_tc(e, hb, db.bv, eo, &tb, /*with_pe=*/false);
  if (s.code != HKB_OK) return s;
  if (!batch->orders) {
    s = finish_orders(e, hb, nullptr, d_orders);
    if (s.code != HKB_OK) return s;
  }
  launch_tf_rows(st, db.bv, d_orders, d_pos, d_rres, e->d_err);
  e->launches += 1;
  HKB_CUDA(cudaEventRecord(e->ev[2], st));
  const F32Weights& w = e->w32;
  for (int l = 0; l < 3; ++l) {
    const std::string q = "dec" + std::to_string(l) + ".";
    // decode weight-stream tile of layer l: [W1a, W1d,] W2, W3, then
    // 4 x (W_in, W_in remainder), then 4 x W_out
    auto tile = [](int layer, int i) { return stream_w2_tile(layer) + i; };
    TfSlotArgs sa;
    sa.bv = db.bv;
    sa.prot_seq0 = d_seq0;
    sa.prot_nseq = d_nseq;
    sa.layer = l;
    sa.h_e = eo.h_e16;
    sa.e_idx = eo.e_idx;
    sa.pos = d_pos;
    sa.tokens = d_tok;
    sa.Aenc0 = tb.Aenc0;
    sa.PVenc = tb.PVenc[l];
    sa.A = A;
    sa.PV = PV;
    sa.Stab = w.dec[l].Stab;
    sa.W1b = e->gemm_img.at(q + "W1b");
    sa.W2 = static_cast<const unsigned char*>(e->d_stream) + (size_t)tile(l, 0) * kTileBytes;
    sa.b2 = w.dec[l].b2;
    sa.S = S;
    sa.err = e->d_err;
    launch_tf_slot_tc(st, sa, e->num_sms);
    TfNodeArgs na;
    na.bv = db.bv;
    na.rows = Q;
    na.layer = l;
    na.row_res = d_rres;
    na.mask = eo.mask;
    na.h_enc = eo.h_v;
    na.h = h;
    na.S = S;
    na.stream = static_cast<const unsigned char*>(e->d_stream);
    na.tile_ids[0] = tile(l, 1);   // W3
    for (int i = 0; i < 4; ++i) {  // the node kernel consumes (W_in, remainder, W_out) per chunk
      na.tile_ids[1 + 3 * i] = tile(l, 2 + 2 * i);
      na.tile_ids[2 + 3 * i] = tile(l, 3 + 2 * i);
      na.tile_ids[3 + 3 * i] = tile(l, 10 + i);
    }
    if (l < 2) {
      na.tile_ids[13] = stream_w1a_tile(l + 1);       // W1a of layer l+1
      na.tile_ids[14] = stream_w1a_tile(l + 1) + 1;   // W1d of layer l+1
      na.b1_next = w.dec[l + 1].b1;
      na.A_next = A;
      na.PV_next = PV;
    }
    const auto& D = w.dec[l];
    na.b3 = D.b3;
    na.n1w = D.n1w;
    na.n1b = D.n1b;
    na.bin = D.bin;
    na.bout = D.bout;
    na.n2w = D.n2w;
    na.n2b = D.n2b;
    na.headT = w.headT;
    na.head_b = w.head_b;
    na.log_probs = LP;
    na.err = e->d_err;
    launch_tf_node_tc(st, na, e->num_sms);
    e->launches += 2;
  }
  launch_scores(st, db.bv, d_tok, LP, eo.mask, sc);
  e->launches += 1;
  HKB_CUDA(cudaEventRecord(e->ev[3], st));
  HKB_CUDA(cudaGetLastError());
  HKB_CUDA(cudaMemcpyAsync(out->log_probs, LP, sizeof(float) * Q * kV, cudaMemcpyDeviceToHost, st));
  if (out->orders)
    HKB_CUDA(cudaMemcpyAsync(out->orders, d_orders, sizeof(int32_t) * Q, cudaMemcpyDeviceToHost,
                             st));
  if (out->scores)
    HKB_CUDA(cudaMemcpyAsync(out->scores, sc, sizeof(float) * hb.NS, cudaMemcpyDeviceToHost, st));
  s = check_device_error(e);
  if (s.code != HKB_OK) return s;
  record_timings(e);
  return kOk;
}

void record_timings(hkb_engine* e) {
  cudaEventElapsedTime(&e->timings[0], e->ev[0], e->ev[1]);
  cudaEventElapsedTime(&e->timings[1], e->ev[1], e->ev[2]);
  cudaEventElapsedTime(&e->timings[2], e->ev[2], e->ev[3]);
  cudaEventElapsedTime(&e->timings[3], e->ev[0], e->ev[3]);
}

}  // namespace
}  // namespace hkb

using namespace hkb;

extern "C" {

int32_t hkb_mpnn_abi_version(void) { return HKB_MPNN_ABI_VERSION; }

hkb_status hkb_mpnn_create(const void* st_blob, size_t length, int device,
                           int32_t precision, hkb_engine** out) {
  if (out == nullptr) return invalid("engine output pointer is null");
  *out = nullptr;
  if (precision != HKB_PRECISION_FP32 && precision != HKB_PRECISION_BF16 &&
      precision != HKB_PRECISION_F16)
    return invalid("precision must be HKB_PRECISION_FP32, HKB_PRECISION_BF16 or HKB_PRECISION_F16");
  std::map<std::string, TensorView> tensors;
  std::vector<float> storage;
  const char* why = nullptr;
  if (!parse_safetensors(st_blob, length, &tensors, &storage, &why)) return invalid(why);
  Prepared P;
  hkb_status s = prepare_f32(tensors, &P);
  if (s.code != HKB_OK) return s;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    cudaGetLastError();
    return {HKB_UNAVAILABLE, "no CUDA device is available"};
  }
  if (device < 0 || device >= ndev) return invalid("device ordinal out of range");
  HKB_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop{};
  HKB_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10) return {HKB_UNAVAILABLE, "this build targets sm_100a (B200) only"};
  auto* e = new hkb_engine();
  e->device = device;
  e->precision = precision;
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&e->d_weights, P.blob.data.size() * sizeof(float)) != cudaSuccess ||
      cudaMalloc((void**)&e->d_err, sizeof(unsigned int)) != cudaSuccess) {
    cudaGetLastError();
    hkb_mpnn_destroy(e);
    return {HKB_UNAVAILABLE, "device allocation failed"};
  }
  e->weights_bytes = P.blob.data.size() * sizeof(float);
  for (auto& ev : e->ev) cudaEventCreate(&ev);
  cudaEventCreateWithFlags(&e->ev_orders, cudaEventDisableTiming);
  cudaEventCreateWithFlags(&e->ev_recheck, cudaEventDisableTiming);
  cudaEventRecord(e->ev_orders, e->stream);
  if (cudaMallocHost(&e->h_recheck, sizeof(unsigned int) * (1 + kRecheckCap)) != cudaSuccess) {
    cudaGetLastError();
    e->h_recheck = nullptr;
    hkb_mpnn_destroy(e);
    return {HKB_UNAVAILABLE, "host allocation failed"};
  }
  // Test hook: HKB_RECHECK_ALL_ORDERS=1 sends every random order through the
  // host recomputation path.
  if (const char* v = std::getenv("HKB_RECHECK_ALL_ORDERS")) e->recheck_all_orders = v[0] == '1';
  // Test hook: the next HKB_STALL_CHECK_CALLS tensor-core design calls run the
  // decode kernel's failure-path check (a bounded wait that runs out).
  if (const char* v = std::getenv("HKB_STALL_CHECK_CALLS")) e->stall_check_calls = std::atoi(v);
  if (cudaMemcpy(e->d_weights, P.blob.data.data(), e->weights_bytes,
                 cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    hkb_mpnn_destroy(e);
    return internal("weight upload failed");
  }
  resolve_f32(P, static_cast<const float*>(e->d_weights), &e->w32);
  std::vector<uint16_t> img;
  if (!build_stream_image(tensors, precision == HKB_PRECISION_F16, &img)) {
    hkb_mpnn_destroy(e);
    return invalid("ProteinMPNN v_48_020 weights: missing decoder tensor");
  }
  if (cudaMalloc(&e->d_stream, img.size() * sizeof(uint16_t)) != cudaSuccess ||
      cudaMemcpy(e->d_stream, img.data(), img.size() * sizeof(uint16_t),
                 cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    hkb_mpnn_destroy(e);
    return {HKB_UNAVAILABLE, "device allocation failed"};
  }
  {
    std::vector<uint16_t> gimg;
    std::map<std::string, size_t> gat;
    if (!build_gemm_images(tensors, &gimg, &gat)) {
      hkb_mpnn_destroy(e);
      return invalid("ProteinMPNN v_48_020 weights: missing tensor");
    }
    if (cudaMalloc(&e->d_gemm, gimg.size() * sizeof(uint16_t)) != cudaSuccess ||
        cudaMemcpy(e->d_gemm, gimg.data(), gimg.size() * sizeof(uint16_t),
                   cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      hkb_mpnn_destroy(e);
      return {HKB_UNAVAILABLE, "device allocation failed"};
    }
    for (const auto& kv : gat)
      e->gemm_img[kv.first] = static_cast<const unsigned char*>(e->d_gemm) + kv.second;
    e->num_sms = prop.multiProcessorCount;
  }
  {
    Bf16DecodeWeights& W = e->wbf;
    W.stream = static_cast<const unsigned char*>(e->d_stream);
    for (int l = 0; l < 3; ++l) {
      const auto& D = e->w32.dec[l];
      W.Stab[l] = D.Stab;
      W.b1[l] = D.b1;
      W.b2[l] = D.b2;
      W.b3[l] = D.b3;
      W.n1w[l] = D.n1w;
      W.n1b[l] = D.n1b;
      W.n2w[l] = D.n2w;
      W.n2b[l] = D.n2b;
      W.bin[l] = D.bin;
      W.bout[l] = D.bout;
    }
    W.headT = e->w32.headT;
    W.head_b = e->w32.head_b;
    // the decode kernel's logit head: [21][kHeadPitch] fp32, rows padded
    auto it = tensors.find("W_out.weight");
    if (it == tensors.end()) {
      hkb_mpnn_destroy(e);
      return invalid("ProteinMPNN v_48_020 weights: missing W_out.weight");
    }
    std::vector<float> hp((size_t)kV * kHeadPitch, 0.0f);
    for (int v = 0; v < kV; ++v)
      for (int f = 0; f < kH; ++f) hp[(size_t)v * kHeadPitch + f] = it->second.data[v * kH + f];
    if (cudaMalloc(&e->d_head, hp.size() * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(e->d_head, hp.data(), hp.size() * sizeof(float), cudaMemcpyHostToDevice) !=
            cudaSuccess) {
      cudaGetLastError();
      hkb_mpnn_destroy(e);
      return {HKB_UNAVAILABLE, "device allocation failed"};
    }
    W.headP = static_cast<const float*>(e->d_head);
  }
  *out = e;
  return kOk;
}

void hkb_mpnn_destroy(hkb_engine* e) {
  if (e == nullptr) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  e->ws.release();
  if (e->d_weights) cudaFree(e->d_weights);
  if (e->d_stream) cudaFree(e->d_stream);
  if (e->d_gemm) cudaFree(e->d_gemm);
  if (e->d_head) cudaFree(e->d_head);
  if (e->d_err) cudaFree(e->d_err);
  for (auto& ev : e->ev)
    if (ev) cudaEventDestroy(ev);
  if (e->ev_orders) cudaEventDestroy(e->ev_orders);
  if (e->ev_recheck) cudaEventDestroy(e->ev_recheck);
  if (e->h_recheck) cudaFreeHost(e->h_recheck);
  if (e->h_orders) cudaFreeHost(e->h_orders);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

hkb_status hkb_mpnn_design(hkb_engine* e, const hkb_design_batch* batch,
                           hkb_design_out* out) {
  if (e == nullptr || batch == nullptr || out == nullptr)
    return invalid("engine, batch and output must be non-null");
  if (out->tokens == nullptr) return invalid("ProteinMPNN inverse-fold output shape is invalid");
  if (batch->num_proteins <= 0 || batch->residue_counts == nullptr)
    return invalid("batch must contain at least one protein");
  if (batch->coords == nullptr || batch->atom_sources == nullptr)
    return invalid("inverse-fold structure must provide canonical backbone atoms");
  HKB_CUDA(cudaSetDevice(e->device));
  int64_t R = 0;
  for (int b = 0; b < batch->num_proteins; ++b) {
    if (batch->residue_counts[b] <= 0)
      return invalid("inverse-fold structure must contain at least one residue");
    R += batch->residue_counts[b];
  }
  if (!finite_coords(batch->coords, batch->atom_sources, R))
    return invalid("coordinates of present atoms must be finite");
  cudaStream_t st = e->stream;
  float* d_coords = e->ws.get_as<float>("in.coords", R * 15);
  uint8_t* d_src = e->ws.get_as<uint8_t>("in.src", R * 5);
  if (!d_coords || !d_src) return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_coords, batch->coords, sizeof(float) * R * 15,
                           cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_src, batch->atom_sources, R * 5, cudaMemcpyHostToDevice, st));
  int64_t Q = 0, NS = 0;
  if (batch->num_seqs == nullptr) return invalid("num_seqs must be non-null");
  for (int b = 0; b < batch->num_proteins; ++b) {
    if (batch->num_seqs[b] <= 0) return invalid("inverse-fold num_seqs must be greater than zero");
    Q += (int64_t)batch->num_seqs[b] * batch->residue_counts[b];
    NS += batch->num_seqs[b];
  }
  DeviceDesignOut o;
  o.tokens = e->ws.get_as<int>("o.tokens", Q);
  o.orders = e->ws.get_as<int>("o.orders", Q);
  o.scores = e->ws.get_as<float>("o.scores", NS);
  // A page-locked, mapped log_probs buffer (cudaHostAlloc / cudaHostRegister)
  // registered against this engine's device is written by the tensor-core
  // decode kernel directly, so its 84 bytes per designed residue cross the
  // bus while the kernel runs instead of in a copy after it; anything else
  // gets a device buffer and a copy.
  bool lp_direct = false;
  if (out->log_probs && e->precision != HKB_PRECISION_FP32) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, out->log_probs) == cudaSuccess &&
        pa.type == cudaMemoryTypeHost && pa.devicePointer != nullptr && pa.device == e->device) {
      o.log_probs = static_cast<float*>(pa.devicePointer);
      lp_direct = true;
    } else {
      (void)cudaGetLastError();   // an unregistered pointer is not an error here
    }
  }
  if (!lp_direct) o.log_probs = e->ws.get_as<float>("o.lp", Q * kV);
  if (!o.tokens || !o.log_probs || !o.orders || !o.scores)
    return {HKB_UNAVAILABLE, "device allocation failed"};
  HostBatch hb;
  hkb_status s = design_common(e, batch, batch->atom_sources, d_coords, d_src, &hb, o);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaMemcpyAsync(out->tokens, o.tokens, sizeof(int) * Q, cudaMemcpyDeviceToHost, st));
  if (out->log_probs && !lp_direct)
    HKB_CUDA(cudaMemcpyAsync(out->log_probs, o.log_probs, sizeof(float) * Q * kV,
                             cudaMemcpyDeviceToHost, st));
  if (out->scores)
    HKB_CUDA(cudaMemcpyAsync(out->scores, o.scores, sizeof(float) * NS,
                             cudaMemcpyDeviceToHost, st));
  if (out->orders)
    HKB_CUDA(cudaMemcpyAsync(out->orders, o.orders, sizeof(int32_t) * Q,
                             cudaMemcpyDeviceToHost, st));
  s = check_device_error(e);
  if (s.code != HKB_OK) return s;
  record_timings(e);
  return kOk;
}

hkb_status hkb_mpnn_design_device(hkb_engine* e, const hkb_design_batch* batch,
                                  hkb_design_out* dout, void* stream) {
  if (e == nullptr || batch == nullptr || dout == nullptr)
    return invalid("engine, batch and output must be non-null");
  if (dout->tokens == nullptr || dout->log_probs == nullptr || dout->orders == nullptr ||
      dout->scores == nullptr)
    return invalid("device design needs tokens, log_probs, orders and scores buffers");
  if (batch->num_proteins <= 0 || batch->residue_counts == nullptr)
    return invalid("batch must contain at least one protein");
  if (batch->coords == nullptr || batch->atom_sources == nullptr)
    return invalid("inverse-fold structure must provide canonical backbone atoms");
  HKB_CUDA(cudaSetDevice(e->device));
  int64_t R = 0;
  for (int b = 0; b < batch->num_proteins; ++b) {
    if (batch->residue_counts[b] <= 0)
      return invalid("inverse-fold structure must contain at least one residue");
    R += batch->residue_counts[b];
  }
  cudaStream_t prev = e->stream;
  if (stream) e->stream = static_cast<cudaStream_t>(stream);
  // The residue mask drives the host-side random orders: read the atom
  // sources back (5 bytes per residue).
  std::vector<uint8_t> host_src((size_t)R * 5);
  cudaError_t ce = cudaMemcpyAsync(host_src.data(), batch->atom_sources, R * 5,
                                   cudaMemcpyDeviceToHost, e->stream);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->stream);
  if (ce != cudaSuccess) {
    e->stream = prev;
    return internal(cudaGetErrorString(ce));
  }
  DeviceDesignOut o{dout->tokens, dout->log_probs, dout->orders, dout->scores};
  HostBatch hb;
  hkb_status s = design_common(e, batch, host_src.data(), batch->coords,
                               batch->atom_sources, &hb, o);
  e->stream = prev;
  return s;
}

hkb_status hkb_mpnn_score(hkb_engine* e, const hkb_score_batch* batch, hkb_score_out* out) {
  if (e == nullptr || batch == nullptr || out == nullptr || out->log_probs == nullptr)
    return invalid("ProteinMPNN teacher-forced output shape is invalid");
  if (batch->num_proteins <= 0 || batch->residue_counts == nullptr ||
      batch->num_seqs == nullptr)
    return invalid("batch must contain at least one protein");
  if (batch->coords == nullptr || batch->atom_sources == nullptr)
    return invalid("ProteinMPNN inverse fold coordinates pointer is null");
  if (batch->tokens == nullptr) return invalid("ProteinMPNN token pointer is null");
  HKB_CUDA(cudaSetDevice(e->device));
  int64_t R = 0;
  for (int b = 0; b < batch->num_proteins; ++b) {
    if (batch->residue_counts[b] <= 0)
      return invalid("inverse-fold structure must contain at least one residue");
    R += batch->residue_counts[b];
  }
  if (!finite_coords(batch->coords, batch->atom_sources, R))
    return invalid("coordinates of present atoms must be finite");
  HostBatch hb;
  hkb_status s = build_host_batch(batch->num_proteins, batch->residue_counts,
                                  batch->num_seqs, batch->atom_sources, &hb);
  if (s.code != HKB_OK) return s;
  for (int64_t q = 0; q < hb.Q; ++q)
    if (batch->tokens[q] < 0 || batch->tokens[q] >= kV)
      return invalid("ProteinMPNN token id is outside the v48 vocabulary");
  hb.seq_seed.resize(hb.NS);
  for (int b = 0; b < hb.B; ++b)
    for (int q = 0; q < hb.S[b]; ++q)
      hb.seq_seed[hb.seq_base[b] + q] = (batch->seeds ? batch->seeds[b] : 0ull) + (uint64_t)q;
  if (e->precision == HKB_PRECISION_F16) {
    if (batch->orders)
      for (int sq = 0; sq < hb.NS; ++sq)
        if (!check_permutation(batch->orders + hb.seq_row_off[sq], hb.L[hb.seq_prot[sq]]))
          return invalid("ProteinMPNN decoding_order must be a permutation");
    return score_tc(e, batch, hb, out);
  }
  if (batch->orders) {
    hb.orders.assign(batch->orders, batch->orders + hb.Q);
    for (int sq = 0; sq < hb.NS; ++sq)
      if (!check_permutation(hb.orders.data() + hb.seq_row_off[sq], hb.L[hb.seq_prot[sq]]))
        return invalid("ProteinMPNN decoding_order must be a permutation");
  } else {
    s = build_orders(nullptr, nullptr, &hb);
    if (s.code != HKB_OK) return s;
  }
  e->launches = 0;
  cudaStream_t st = e->stream;
  HKB_CUDA(cudaMemsetAsync(e->d_err, 0, sizeof(unsigned int), st));
  float* d_coords = e->ws.get_as<float>("in.coords", R * 15);
  uint8_t* d_src = e->ws.get_as<uint8_t>("in.src", R * 5);
  if (!d_coords || !d_src) return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_coords, batch->coords, sizeof(float) * R * 15,
                           cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_src, batch->atom_sources, R * 5, cudaMemcpyHostToDevice, st));
  DeviceBatch db;
  db.coords = d_coords;
  db.sources = d_src;
  s = upload_tables(e, hb, &db);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[0], st));
  EncoderOut eo;
  s = encode_f32(e, hb, db, &eo);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[1], st));
  DecoderTables dt{};
  s = decoder_tables_f32(e, hb, eo, &dt);
  if (s.code != HKB_OK) return s;
  HKB_CUDA(cudaEventRecord(e->ev[2], st));
  // Teacher-forced pass in chunks of whole sequences.
  const F32Weights& w = e->w32;
  const int64_t kChunkRows = 16384;
  int sq0 = 0;
  std::vector<float> host_lp((size_t)hb.Q * kV);
  while (sq0 < hb.NS) {
    int sq1 = sq0;
    int64_t rows = 0;
    while (sq1 < hb.NS && (rows == 0 || rows + hb.L[hb.seq_prot[sq1]] <= kChunkRows)) {
      rows += hb.L[hb.seq_prot[sq1]];
      ++sq1;
    }
    std::vector<int> row_res(rows), row_prot(rows), pos(rows), toks(rows);
    std::vector<int64_t> row_base(rows);
    int64_t at = 0;
    const int64_t qbase = hb.seq_row_off[sq0];
    for (int sq = sq0; sq < sq1; ++sq) {
      const int b = hb.seq_prot[sq];
      const int64_t q0 = hb.seq_row_off[sq];
      for (int t = 0; t < hb.L[b]; ++t) {
        row_res[at + t] = hb.off[b] + t;
        row_prot[at + t] = b;
        row_base[at + t] = at;
        toks[at + t] = batch->tokens[q0 + t];
      }
      for (int p = 0; p < hb.L[b]; ++p) pos[at + hb.orders[q0 + p]] = p;
      at += hb.L[b];
    }
    int* d_rr = e->ws.get_as<int>("tf.rr", rows);
    int* d_rp = e->ws.get_as<int>("tf.rp", rows);
    int* d_pos = e->ws.get_as<int>("tf.pos", rows);
    int* d_tok = e->ws.get_as<int>("tf.tok", rows);
    int64_t* d_rb = e->ws.get_as<int64_t>("tf.rb", rows);
    float* h = e->ws.get_as<float>("tf.h", rows * kH);
    float* AP = e->ws.get_as<float>("tf.AP", rows * 256);
    float* G1 = e->ws.get_as<float>("tf.G1", rows * kK * kH);
    float* G2 = e->ws.get_as<float>("tf.G2", rows * kK * kH);
    float* Sv = e->ws.get_as<float>("tf.S", rows * kH);
    float* kc = e->ws.get_as<float>("tf.kc", rows);
    float* T3 = e->ws.get_as<float>("tf.T3", rows * kH);
    float* h1 = e->ws.get_as<float>("tf.h1", rows * kH);
    float* F = e->ws.get_as<float>("tf.F", rows * kFfn);
    float* Y = e->ws.get_as<float>("tf.Y", rows * kH);
    float* Z = e->ws.get_as<float>("tf.Z", rows * kV);
    float* LP = e->ws.get_as<float>("tf.LP", rows * kV);
    if (!d_rr || !d_rp || !d_pos || !d_tok || !d_rb || !h || !AP || !G1 || !G2 || !Sv ||
        !kc || !T3 || !h1 || !F || !Y || !Z || !LP)
      return {HKB_UNAVAILABLE, "device allocation failed"};
    HKB_CUDA(cudaMemcpyAsync(d_rr, row_res.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, st));
    HKB_CUDA(cudaMemcpyAsync(d_rp, row_prot.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, st));
    HKB_CUDA(cudaMemcpyAsync(d_pos, pos.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, st));
    HKB_CUDA(cudaMemcpyAsync(d_tok, toks.data(), sizeof(int) * rows, cudaMemcpyHostToDevice, st));
    HKB_CUDA(cudaMemcpyAsync(d_rb, row_base.data(), sizeof(int64_t) * rows, cudaMemcpyHostToDevice, st));
    TfRows tr;
    tr.rows = rows;
    tr.row_res = d_rr;
    tr.row_seqbase = d_rb;
    tr.row_prot = d_rp;
    tr.pos = d_pos;
    tr.tokens = d_tok;
    launch_gather_rows(st, rows, d_rr, eo.h_v, h);
    e->launches += 1;
    for (int l = 0; l < 3; ++l) {
      const auto& D = w.dec[l];
      gemm_f32(st, rows, 256, kH, h, kH, D.W1adT, 256, D.b1ad, 0, AP, 256);
      launch_tf_slot_in(st, db.bv, tr, l, AP, dt, D.Stab, eo.e_idx, G1);
      gemm_f32(st, rows * kK, kH, kH, G1, kH, D.W2T, kH, D.b2, 1, G2, kH);
      launch_row_slot_sum(st, db.bv, tr, G2, Sv, kc);
      gemm_f32(st, rows, kH, kH, Sv, kH, D.W3T, kH, nullptr, 0, T3, kH);
      launch_dec_node_update(st, rows, T3, kc, D.b3, h, D.n1w, D.n1b, h1);
      gemm_f32(st, rows, kFfn, kH, h1, kH, D.WinT, kFfn, D.bin, 1, F, kFfn);
      gemm_f32(st, rows, kH, kFfn, F, kFfn, D.WoutT, kH, nullptr, 0, Y, kH);
      launch_ln_rows(st, rows, h1, Y, D.bout, D.n2w, D.n2b, eo.mask, d_rr, h);
      e->launches += 9;
    }
    gemm_f32(st, rows, kV, kH, h, kH, w.headT, kV, w.head_b, 0, Z, kV);
    launch_log_softmax_rows(st, rows, Z, LP);
    e->launches += 2;
    HKB_CUDA(cudaMemcpyAsync(host_lp.data() + qbase * kV, LP, sizeof(float) * rows * kV,
                             cudaMemcpyDeviceToHost, st));
    HKB_CUDA(cudaStreamSynchronize(st));
    sq0 = sq1;
  }
  HKB_CUDA(cudaEventRecord(e->ev[3], st));
  s = check_device_error(e);
  if (s.code != HKB_OK) return s;
  record_timings(e);
  std::memcpy(out->log_probs, host_lp.data(), sizeof(float) * hb.Q * kV);
  if (out->orders) std::memcpy(out->orders, hb.orders.data(), sizeof(int32_t) * hb.Q);
  if (out->scores) {
    for (int sq = 0; sq < hb.NS; ++sq) {
      const int b = hb.seq_prot[sq];
      const int64_t q0 = hb.seq_row_off[sq];
      double loss = 0.0, cnt = 0.0;
      for (int t = 0; t < hb.L[b]; ++t) {
        const float m = hb.mask[hb.off[b] + t];
        if (m == 0.0f) continue;
        loss -= (double)host_lp[(q0 + t) * kV + batch->tokens[q0 + t]];
        cnt += (double)m;
      }
      out->scores[sq] = cnt > 0.0 ? (float)(loss / cnt) : 0.0f;
    }
  }
  return kOk;
}

static hkb_status single_protein_encode(hkb_engine* e, int32_t L, const float* coords,
                                        const uint8_t* src, HostBatch* hb, DeviceBatch* db,
                                        EncoderOut* eo, bool full) {
  if (e == nullptr) return invalid("engine is null");
  if (L <= 0) return invalid("inverse-fold structure must contain at least one residue");
  if (coords == nullptr || src == nullptr)
    return invalid("inverse-fold structure must provide canonical backbone atoms");
  if (!finite_coords(coords, src, L)) return invalid("coordinates of present atoms must be finite");
  HKB_CUDA(cudaSetDevice(e->device));
  const int32_t one = 1;
  hkb_status s = build_host_batch(1, &L, &one, src, hb);
  if (s.code != HKB_OK) return s;
  cudaStream_t st = e->stream;
  e->launches = 0;
  HKB_CUDA(cudaMemsetAsync(e->d_err, 0, sizeof(unsigned int), st));
  float* d_coords = e->ws.get_as<float>("in.coords", (size_t)L * 15);
  uint8_t* d_src = e->ws.get_as<uint8_t>("in.src", (size_t)L * 5);
  if (!d_coords || !d_src) return {HKB_UNAVAILABLE, "device allocation failed"};
  HKB_CUDA(cudaMemcpyAsync(d_coords, coords, sizeof(float) * L * 15, cudaMemcpyHostToDevice, st));
  HKB_CUDA(cudaMemcpyAsync(d_src, src, (size_t)L * 5, cudaMemcpyHostToDevice, st));
  db->coords = d_coords;
  db->sources = d_src;
  s = upload_tables(e, *hb, db);
  if (s.code != HKB_OK) return s;
  if (full)
    return e->precision == HKB_PRECISION_F16 ? encode_tc(e, *hb, *db, eo)
                                             : encode_f32(e, *hb, *db, eo);
  eo->e_idx = e->ws.get_as<int>("e.idx", (size_t)L * kK);
  eo->d2 = e->ws.get_as<float>("e.d2", (size_t)L * kK);
  eo->mask = e->ws.get_as<float>("e.mask", L);
  if (!eo->e_idx || !eo->d2 || !eo->mask) return {HKB_UNAVAILABLE, "device allocation failed"};
  launch_knn(st, db->bv, d_coords, d_src, eo->e_idx, eo->d2, eo->mask, e->d_err, L);
  e->launches += 1;
  HKB_CUDA(cudaGetLastError());
  return kOk;
}


static void compact_rows(const void* src, void* dst, int L, int K, size_t elem, size_t width) {
  // [L,48,width] -> [L,K,width]
  for (int i = 0; i < L; ++i)
    std::memcpy(static_cast<char*>(dst) + (size_t)i * K * width * elem,
                static_cast<const char*>(src) + (size_t)i * kK * width * elem,
                (size_t)K * width * elem);
}

hkb_status hkb_mpnn_encode(hkb_engine* e, int32_t L, const float* coords,
                           const uint8_t* src, float* h_v, float* h_e, int32_t* e_idx) {
  HostBatch hb;
  DeviceBatch db;
  EncoderOut eo;
  hkb_status s = single_protein_encode(e, L, coords, src, &hb, &db, &eo, true);
  if (s.code != HKB_OK) return s;
  const int K = std::min(L, kK);
  std::vector<float> he((size_t)L * kK * kH);
  std::vector<uint16_t> he16(eo.h_e16 ? he.size() : 0), he16lo(he16.size());
  std::vector<int> idx((size_t)L * kK);
  cudaStream_t st = e->stream;
  if (h_v) HKB_CUDA(cudaMemcpyAsync(h_v, eo.h_v, sizeof(float) * L * kH, cudaMemcpyDeviceToHost, st));
  if (eo.h_e16) {
    HKB_CUDA(cudaMemcpyAsync(he16.data(), eo.h_e16, he16.size() * sizeof(uint16_t),
                             cudaMemcpyDeviceToHost, st));
    HKB_CUDA(cudaMemcpyAsync(he16lo.data(), eo.h_e16lo, he16lo.size() * sizeof(uint16_t),
                             cudaMemcpyDeviceToHost, st));
  }
  else
    HKB_CUDA(cudaMemcpyAsync(he.data(), eo.h_e, he.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
  HKB_CUDA(cudaMemcpyAsync(idx.data(), eo.e_idx, idx.size() * sizeof(int), cudaMemcpyDeviceToHost, st));
  s = check_device_error(e);
  if (s.code != HKB_OK) return s;
  for (size_t i = 0; i < he16.size(); ++i) he[i] = half_to_float(he16[i]) + half_to_float(he16lo[i]);
  if (h_e) compact_rows(he.data(), h_e, L, K, sizeof(float), kH);
  if (e_idx) compact_rows(idx.data(), e_idx, L, K, sizeof(int), 1);
  return kOk;
}

hkb_status hkb_mpnn_knn(hkb_engine* e, int32_t L, const float* coords, const uint8_t* src,
                        int32_t* e_idx, float* d2) {
  if (e_idx == nullptr) return invalid("e_idx output pointer is null");
  HostBatch hb;
  DeviceBatch db;
  EncoderOut eo;
  hkb_status s = single_protein_encode(e, L, coords, src, &hb, &db, &eo, false);
  if (s.code != HKB_OK) return s;
  const int K = std::min(L, kK);
  std::vector<float> dd((size_t)L * kK);
  std::vector<int> idx((size_t)L * kK);
  cudaStream_t st = e->stream;
  HKB_CUDA(cudaMemcpyAsync(dd.data(), eo.d2, dd.size() * sizeof(float), cudaMemcpyDeviceToHost, st));
  HKB_CUDA(cudaMemcpyAsync(idx.data(), eo.e_idx, idx.size() * sizeof(int), cudaMemcpyDeviceToHost, st));
  s = check_device_error(e);
  if (s.code != HKB_OK) return s;
  compact_rows(idx.data(), e_idx, L, K, sizeof(int), 1);
  if (d2) compact_rows(dd.data(), d2, L, K, sizeof(float), 1);
  return kOk;
}

int64_t hkb_mpnn_last_launch_count(const hkb_engine* e) { return e ? e->launches : -1; }

hkb_status hkb_mpnn_last_timings(const hkb_engine* e, float* ms4) {
  if (e == nullptr || ms4 == nullptr) return invalid("engine and output must be non-null");
  // Phases are bracketed by events on the launching stream; read them once
  // the call's work has completed.
  const int pairs[4][2] = {{0, 1}, {1, 2}, {2, 3}, {0, 3}};
  for (int i = 0; i < 4; ++i) {
    float ms = 0.0f;
    const cudaError_t ce = cudaEventElapsedTime(&ms, e->ev[pairs[i][0]], e->ev[pairs[i][1]]);
    if (ce != cudaSuccess) {
      cudaGetLastError();
      return {HKB_FAILED_PRECONDITION, cudaGetErrorString(ce)};
    }
    ms4[i] = ms;
  }
  return kOk;
}

}  // extern "C"
