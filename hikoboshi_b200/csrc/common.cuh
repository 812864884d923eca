// Shared device-side definitions for the ProteinMPNN v_48_020 design engine.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace hkb {

constexpr int kH = 128;         // hidden width
constexpr int kK = 48;          // neighbours per residue (max)
constexpr int kV = 21;          // vocabulary "ACDEFGHIKLMNPQRSTVWYX"
constexpr int kFfn = 512;       // FFN hidden
constexpr int kEdgeIn = 416;    // 16 positional + 25 pairs x 16 RBF
constexpr int kRbf = 16;
constexpr int kPairs = 25;
constexpr int kPosClasses = 66;
constexpr float kMessageScale = 30.0f;
constexpr float kLnEps = 1.0e-5f;

// Device error word bits (read by the host after each call; kernels never
// trap, they record and return).
enum DeviceError : unsigned int {
  kErrNone = 0,
  kErrBadIndex = 1u << 0,
  kErrTimeout = 1u << 1,
  kErrTmemAlloc = 1u << 2,
};

// exp(x) for x <= 0: integer range reduction against e^-n (n = 0..16) and a
// 6th-order Taylor polynomial for the remainder r in [-0.5, 0.5]; 0 below -16
// (the reference's rule, cpp/include/hikoboshi/primitives/detail/
// fast_exp_neg.hpp:9-52).  The table holds e^-n rounded to float.
static __constant__ float c_exp_neg_table[17] = {
    1.0f, 0.3678794503211975f, 0.1353352814912796f, 0.049787066876888275f,
    0.018315639346837997f, 0.0067379469983279705f, 0.0024787522852420807f,
    0.0009118819725699723f, 0.000335462624207139f, 0.00012340980174485594f,
    4.539993096841499e-05f, 1.6701700587873347e-05f, 6.1442124206223525e-06f,
    2.260329438286135e-06f, 8.315287232107949e-07f, 3.0590231858695915e-07f,
    1.1253517584464134e-07f};

__device__ __forceinline__ float exp_neg(float x) {
  if (x != x) return x;
  float nx = -x;
  if (nx > 16.0f) return 0.0f;
  if (nx < 0.0f) nx = 0.0f;
  int n = __float2int_rz(__fadd_rn(nx, 0.5f));
  if (n > 16) n = 16;
  const float r = -__fsub_rn(nx, (float)n);
  float p = __fadd_rn(1.0f / 120.0f, __fmul_rn(r, 1.0f / 720.0f));
  p = __fadd_rn(1.0f / 24.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f / 6.0f, __fmul_rn(r, p));
  p = __fadd_rn(0.5f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  p = __fadd_rn(1.0f, __fmul_rn(r, p));
  return __fmul_rn(c_exp_neg_table[n], p);
}

// The 25 (query atom, neighbour atom) slot pairs of the RBF block, in the
// reference's order (atom_pair_distance_scalar.cpp:21-72); slot order N=0
// CA=1 C=2 O=3 CB=4.
static __constant__ unsigned char c_pairs[25][2] = {
    {1, 1}, {0, 0}, {2, 2}, {3, 3}, {4, 4}, {1, 0}, {1, 2}, {1, 3}, {1, 4},
    {0, 2}, {0, 3}, {0, 4}, {4, 2}, {4, 3}, {3, 2}, {0, 1}, {2, 1}, {3, 1},
    {4, 1}, {2, 0}, {3, 0}, {4, 0}, {2, 4}, {3, 4}, {2, 3}};

// sqrt(|x_j - x_i|^2 + 1e-6) with the reference's operation order
// (atom_pair_distance_scalar.cpp:122-164), every step correctly rounded.
__device__ __forceinline__ float pair_distance(const float* xi, const float* xj) {
  float sq = 0.0f;
#pragma unroll
  for (int x = 0; x < 3; ++x) {
    const float dl = __fsub_rn(xj[x], xi[x]);
    sq = __fadd_rn(sq, __fmul_rn(dl, dl));
  }
  return __fsqrt_rn(__fadd_rn(sq, 1.0e-6f));
}

// RBF f of 16 on centres linspace(2, 22), sigma = 20 / (16 / sqrt(1/2))
// (rbf_scalar.cpp:10-35, edge_rbf_features_scalar.cpp:135-137).
__device__ __forceinline__ float rbf_value(float dist, int f) {
  const float sigma = (22.0f - 2.0f) / (16.0f / 0.7071067811865475f);
  const float two_s2 = 2.0f * sigma * sigma;
  const float step = (22.0f - 2.0f) / 15.0f;
  const float c = __fadd_rn(2.0f, __fmul_rn((float)f, step));
  const float dl = __fsub_rn(dist, c);
  return exp_neg(__fdiv_rn(-__fmul_rn(dl, dl), two_s2));
}

// GELU(x) = x/2 (1 + erf(x / sqrt 2)), erf by Abramowitz & Stegun 7.1.26
// with exp(-v^2) from exp_neg (reference: cpp/include/hikoboshi/primitives/
// compute/gelu.hpp:22-51).  Used by the fp32 parity path.
__device__ __forceinline__ float gelu_as(float x) {
  float v = x * 0.7071067811865475f;
  float sign = 1.0f;
  if (v < 0.0f) {
    sign = -1.0f;
    v = -v;
  }
  float e;
  if (v > 4.0f) {
    e = sign;
  } else {
    const float t = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(0.3275911f, v)));
    float p = 1.061405429f * t + -1.453152027f;
    p = p * t + 1.421413741f;
    p = p * t + -0.284496736f;
    p = p * t + 0.254829592f;
    p = p * t;
    e = sign * (1.0f - p * exp_neg(-(v * v)));
  }
  return 0.5f * x * (1.0f + e);
}

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU(x) ~= x/2 (1 + tanh(u(x))) with u an odd degree-5 polynomial fitted to
// the exact erf form: max error 2.5e-5 with exact tanh, against 4.7e-4 for
// the textbook cubic u, whose error is one-signed over wide ranges and so
// accumulates through the 48-slot sums.  x^2 is clamped to 25 inside the
// polynomial: for |x| > 5 that gives |u| >= 1.50 |x| > 7.5, where tanh has
// saturated.  tanh is the hardware tanh.approx.f32.  gelu2_tc returns twice
// the value (x (1 + tanh u)), for sums that halve once at the end.  The fp32
// parity path uses the reference's erf form instead (gelu_as).
__device__ __forceinline__ float gelu2_tc(float x) {
  const float x2 = fminf(x * x, 25.0f);
  const float u = x * fmaf(fmaf(-3.51516790e-04f, x2, 3.70056460e-02f), x2, 7.97507884e-01f);
  return fmaf(x, tanh_approx(u), x);
}
__device__ __forceinline__ float gelu_tc(float x) { return 0.5f * gelu2_tc(x); }

// gelu2_tc on two values at once through the packed fp32 pipe (mul / fma
// .f32x2): each lane takes the same roundings in the same order as the scalar
// form, so the results are identical, at about half the FP32 issue slots.
__device__ __forceinline__ float2 gelu2_tc_x2(const float2 x) {
  float2 x2 = __fmul2_rn(x, x);
  x2.x = fminf(x2.x, 25.0f);
  x2.y = fminf(x2.y, 25.0f);
  float2 p = __ffma2_rn(make_float2(-3.51516790e-04f, -3.51516790e-04f), x2,
                        make_float2(3.70056460e-02f, 3.70056460e-02f));
  p = __ffma2_rn(p, x2, make_float2(7.97507884e-01f, 7.97507884e-01f));
  const float2 u = __fmul2_rn(x, p);
  return __ffma2_rn(x, make_float2(tanh_approx(u.x), tanh_approx(u.y)), x);
}

// GELU itself on two values (half of gelu2_tc_x2, an exact scaling).
__device__ __forceinline__ float2 gelu_tc_x2(const float2 x) {
  return __fmul2_rn(gelu2_tc_x2(x), make_float2(0.5f, 0.5f));
}

// 16-byte asynchronous global -> shared copies (cp.async, L2 only).  With
// pred false nothing is read and the 16 bytes are zero-filled.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
// waits until at most one committed group is still in flight
__device__ __forceinline__ void cp_async_wait_one() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// LayerNorm of a 128-wide row held 4 values per lane by one warp:
// two-pass mean / population variance, eps 1e-5 (reference semantics:
// cpp/primitives/compute/layer_norm_scalar.cpp:8-40 computes the same
// statistics with Welford's update).
// g and b are 16-byte aligned rows of 128 (every weight row is).
__device__ __forceinline__ void warp_layer_norm128(float (&x)[4], const float* g,
                                                  const float* b, int lane) {
  const float4 gv = reinterpret_cast<const float4*>(g)[lane];   // in flight during the sums
  const float4 bv = reinterpret_cast<const float4*>(b)[lane];
  float s = warp_sum(x[0] + x[1] + x[2] + x[3]);
  const float mean = s * (1.0f / 128.0f);
  float d0 = x[0] - mean, d1 = x[1] - mean, d2 = x[2] - mean, d3 = x[3] - mean;
  float v = warp_sum(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3) * (1.0f / 128.0f);
  const float inv = 1.0f / sqrtf(v + kLnEps);
  x[0] = d0 * inv * gv.x + bv.x;
  x[1] = d1 * inv * gv.y + bv.y;
  x[2] = d2 * inv * gv.z + bv.z;
  x[3] = d3 * inv * gv.w + bv.w;
}

}  // namespace hkb
