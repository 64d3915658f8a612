// Deterministic stochastic rounding of network weights to a 16-bit tensor-core
// operand format (fp16 or bf16), used once per weight load by the pack kernels.
//
// Rounding to nearest maps a weight w to the closer 16-bit neighbour.  After
// an optimiser step every weight moves by about the learning rate, and when
// that step is comparable to the 16-bit spacing round-to-nearest shortens or
// lengthens all of the steps of one binade in the same direction: a bias
// coherent with the gradient that the network outputs sum up.  Stochastic
// rounding makes the rounded weight unbiased (E[round(w)] = w) so those
// errors stay uncorrelated.  The random choice is a pure function of the
// weight's index in the weight blob, so a pack is reproducible and a CPU model
// can repeat it bit for bit.
//
// Rule, for a weight x (fp32) with index i in the blob:
//   n = x rounded to nearest (even) in the format; if n == x (or n is not
//   finite) the result is n.  Otherwise o is the other format neighbour of x
//   (on the far side of x from n), d = |x - n|, g = |o - n| (a power of two),
//   u = mix32(i) in [0, 2^32).  The result is o when d * 2^32 > u * g, else n,
//   so o is taken with probability d / g.  Both products are exact in double.
// mix32 is the "lowbias32" integer hash published by Chris Wellons
// (xorshift-multiply, two rounds).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace gz {

__host__ __device__ __forceinline__ uint32_t mix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

template <typename T> struct Fmt16;
template <> struct Fmt16<__half> {
  static __device__ __forceinline__ uint16_t rn(float x) { return __half_as_ushort(__float2half_rn(x)); }
  static __device__ __forceinline__ float value(uint16_t b) { return __half2float(__ushort_as_half(b)); }
};
template <> struct Fmt16<__nv_bfloat16> {
  static __device__ __forceinline__ uint16_t rn(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ float value(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
};

// The 16-bit pattern of weight x (blob index i), stochastically rounded.
template <typename T>
__device__ __forceinline__ uint16_t weight_bits_sr(float x, uint32_t i) {
  const uint16_t nb = Fmt16<T>::rn(x);
  const float n = Fmt16<T>::value(nb);
  if (n == x || !isfinite(n)) return nb;
  const bool up = x > n;  // o lies above n
  uint16_t ob;
  if ((nb & 0x7FFF) == 0) ob = up ? 0x0001 : 0x8001;  // from a zero to the smallest value of x's sign
  else ob = (up != ((nb & 0x8000) != 0)) ? (uint16_t)(nb + 1) : (uint16_t)(nb - 1);  // |o| > |n| iff moving away from 0
  const double d = fabs((double)x - (double)n), g = fabs((double)Fmt16<T>::value(ob) - (double)n);
  return d * 4294967296.0 > (double)mix32(i) * g ? ob : nb;
}

}  // namespace gz
