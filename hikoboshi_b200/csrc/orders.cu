// Decoding orders on the device, one CTA per sequence.
//
// The random order (cpp/modules/mpnn/decode_order_scalar.cpp:21-42, 89-116)
// sorts residues by score_r = (mask_r + 1e-4f) * z_r, ties by residue index,
// where z_r = (float)|sqrt(-2 ln u1) cos(2 pi u2)| and u1, u2 are draws 2r and
// 2r+1 of a SplitMix64 stream seeded with the sequence seed.  SplitMix64's
// state after k draws is seed + k * 0x9E3779B97F4A7C15, so every residue's
// draws are computed independently; the sort is a rank count against the
// other scores in shared memory (exact, O(L^2 / threads)).
//
// Exactness.  The reference computes z in double with the host libm and
// rounds it to float.  This kernel calls the device's double log, cos and
// sqrt.  sqrt is correctly rounded on both sides; the device log and cos are
// within 1 and 2 ulp of the true value, the host's within 1 ulp, so the two
// double values of |radius * cos(.)| differ by a few double ulps at most.
// They round to the same float unless the device value lies close to a float
// rounding midpoint: its 29 low mantissa bits (the bits a double -> float
// conversion drops) within kMidpointUlps of 2^28.  Such a residue (about 1 in
// 10^6) marks its sequence, and the host recomputes that sequence's order with
// the host libm, the reference's exact arithmetic, before the decode reads it.
// All float operations after the cast are single correctly rounded float ops
// in the reference's order.
#include "common.cuh"
#include "kernels.hpp"

namespace hkb {
namespace {

constexpr int kOrderThreads = 256;
constexpr uint64_t kMidpointUlps = 256;

__device__ __forceinline__ uint64_t splitmix_at(uint64_t seed, uint64_t k) {
  // output of draw k (0-based): state advanced k + 1 times
  uint64_t z = seed + (k + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(kOrderThreads) decode_order_kernel(OrderArgs a) {
  __shared__ float score[kMaxResidues];
  __shared__ int near_flag;
  const int sq = blockIdx.x;
  const int b = a.bv.seq_prot[sq];
  const int L = a.bv.prot_len[b];
  const int off = a.bv.prot_res_off[b];
  const int64_t row = a.bv.seq_row_off[sq];
  const int mode = a.modes ? a.modes[b] : 0;
  int32_t* order = a.orders + row;
  if (L <= 0 || L > kMaxResidues) {
    if (threadIdx.x == 0) atomicOr(a.err, kErrBadIndex);
    return;
  }
  if (mode == 1) {   // N_TO_C: identity
    for (int p = threadIdx.x; p < L; p += kOrderThreads) order[p] = p;
    return;
  }
  if (mode == 2) {   // INPUT: the caller's permutation (validated on the host)
    for (int p = threadIdx.x; p < L; p += kOrderThreads) order[p] = a.input_orders[off + p];
    return;
  }
  if (threadIdx.x == 0) near_flag = 0;
  __syncthreads();
  const uint64_t seed = a.seeds[sq];
  bool near = false;
  for (int r = threadIdx.x; r < L; r += kOrderThreads) {
    double u1 = (double)(splitmix_at(seed, 2ull * r) >> 11) * (1.0 / 9007199254740992.0);
    if (u1 <= 0.0) u1 = 1.0 / 9007199254740992.0;
    const double u2 = (double)(splitmix_at(seed, 2ull * r + 1) >> 11) * (1.0 / 9007199254740992.0);
    const double radius = sqrt(__dmul_rn(-2.0, log(u1)));
    const double v = fabs(__dmul_rn(radius, cos(__dmul_rn(6.283185307179586476925286766559, u2))));
    const uint64_t low = (uint64_t)__double_as_longlong(v) & ((1ull << 29) - 1);
    const uint64_t mid = 1ull << 28;
    if ((low > mid ? low - mid : mid - low) <= kMidpointUlps) near = true;
    const float z = __double2float_rn(v);
    const uint8_t* s = a.sources + (int64_t)(off + r) * 5;
    const float m = (s[0] && s[1] && s[2] && s[3]) ? 1.0f : 0.0f;
    score[r] = __fmul_rn(__fadd_rn(m, 0.0001f), z);
  }
  if (near || a.recheck_all) near_flag = 1;
  __syncthreads();
  for (int r = threadIdx.x; r < L; r += kOrderThreads) {
    const float sr = score[r];
    int rank = 0;
    for (int j = 0; j < L; ++j) {
      const float sj = score[j];
      rank += (sj < sr || (sj == sr && j < r)) ? 1 : 0;
    }
    order[rank] = r;
  }
  if (threadIdx.x == 0 && near_flag) {
    const unsigned int i = atomicAdd(a.recheck_count, 1u);
    if (i < (unsigned int)a.recheck_cap) a.recheck_list[i] = sq;
  }
}

}  // namespace

void launch_decode_orders(cudaStream_t st, const OrderArgs& a) {
  if (a.bv.num_sequences <= 0) return;
  decode_order_kernel<<<a.bv.num_sequences, kOrderThreads, 0, st>>>(a);
}

}  // namespace hkb
