// numpy's float32 arithmetic for the reference's host sampler, restated for the device.
//
// The reference samples every decision on the host in numpy float32
// (cardgym/rl/ppo.py:75-94): exp of the legal-max-shifted logits, a last-axis sum, one
// division per entry, a running cumsum compared with a float64 uniform. Matching its draws
// bit for bit needs numpy's own exp and its own summation order, both restated here.
//
// numpy 2.3 (the version in this image), x86-64 hosts with AVX2+FMA3 or AVX-512F:
// np.exp on float32 dispatches to the SIMD routine of
// numpy/_core/src/umath/loops_exponent_log.dispatch.c.src. Its published method:
//   k = rint(x * log2(e)); r = x - k * ln2 in two fused steps (a Cody-Waite split of ln 2);
//   exp(r) ~ P(r) / Q(r), P of degree 5 and Q of degree 2 (a minimax rational fit);
//   result = (P / Q) * 2^k, with x >= 88.7228... -> +inf, x <= -103.972... -> 0, NaN kept.
// The coefficients below are that routine's float32 constants; the restatement was checked
// here against np.exp on every float32 in [-104, 0] (1,120,927,745 inputs, zero
// differences, the AVX2 and AVX-512F paths agreeing). Hosts without AVX2/FMA3 fall back to
// libm's expf, which this does not reproduce.
//
// numpy's add-reduction of a contiguous float32 row is pairwise_sum
// (numpy/_core/src/umath/loops_utils.h.src) started from the identity 0: rows shorter than
// 8 add in order; up to 128 elements, eight running sums over the columns i mod 8 of the
// first n - n % 8 entries, combined as ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)),
// then the n % 8 tail in order; longer rows split at n / 2 rounded down to a multiple of 8
// and add the two halves' sums.
//
// Every operation is written with an explicit round-to-nearest intrinsic so that the
// compiler cannot contract or reorder it.
#pragma once

#include <cuda_runtime.h>

namespace cg {

namespace numpy_f32 {
constexpr float kLog2e = 0x1.715476p+0f;
constexpr float kLn2Hi = -6.93145752e-1f;
constexpr float kLn2Lo = -1.42860677e-6f;
constexpr float kP0 = 9.999999999980870924916e-01f;
constexpr float kP1 = 7.257664613233124478488e-01f;
constexpr float kP2 = 2.473615434895520810817e-01f;
constexpr float kP3 = 5.114512081637298353406e-02f;
constexpr float kP4 = 6.757896990527504603057e-03f;
constexpr float kP5 = 5.082762800157070e-04f;
constexpr float kQ1 = -2.742335390411667452936e-01f;
constexpr float kQ2 = 2.159509375685829852307e-02f;
constexpr float kXMax = 88.72283935546875f;
constexpr float kXMin = -103.97208404541015625f;
}  // namespace numpy_f32

// value * 2^k for value in [0.5, 2) and k in [-151, 128], rounded once (as ldexp does).
__device__ __forceinline__ float scale_by_pow2(float value, int k) {
  if (k > 127) return __fmul_rn(__fmul_rn(value, 0x1p127f), __int_as_float(((k - 127) + 127) << 23));
  if (k >= -126) return __fmul_rn(value, __int_as_float((k + 127) << 23));
  // Subnormal result: an exact step to 2^-64 first, then the one rounding multiply.
  return __fmul_rn(__fmul_rn(value, 0x1p-64f), __int_as_float((k + 64 + 127) << 23));
}

__device__ __forceinline__ float numpy_expf(float x) {
  using namespace numpy_f32;
  if (x != x) return x;
  if (x >= kXMax) return __int_as_float(0x7f800000);
  if (x <= kXMin) return 0.f;
  const float k = rintf(__fmul_rn(x, kLog2e));
  float r = __fmaf_rn(k, kLn2Hi, x);
  r = __fmaf_rn(k, kLn2Lo, r);
  float num = __fmaf_rn(kP5, r, kP4);
  num = __fmaf_rn(num, r, kP3);
  num = __fmaf_rn(num, r, kP2);
  num = __fmaf_rn(num, r, kP1);
  num = __fmaf_rn(num, r, kP0);
  float den = __fmaf_rn(kQ2, r, kQ1);
  den = __fmaf_rn(den, r, 1.0f);
  return scale_by_pow2(__fdiv_rn(num, den), static_cast<int>(k));
}

// numpy's pairwise block for 8 <= n <= 128 (see above); every lane of the warp calls it and
// every lane gets the sum. `v` is readable by the whole warp (shared memory).
__device__ __forceinline__ float numpy_block_sum(const float* v, int n) {
  const int lane = threadIdx.x & 31;
  const int body = n - n % 8;
  float r = 0.f;
  if (lane < 8) {
    r = v[lane];
    for (int i = 8 + lane; i < body; i += 8) r = __fadd_rn(r, v[i]);
  }
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
  r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
  float total = __shfl_sync(0xffffffffu, r, 0);
  for (int i = body; i < n; ++i) total = __fadd_rn(total, v[i]);
  return total;
}

// numpy's float32 sum of a contiguous row of n <= kNumpySumMax entries (three levels of
// halving bring any such row down to blocks of at most 128). Called by a whole warp; the
// result is the same in every lane.
constexpr int kNumpySumMax = 512;

template <int kDepth = 3>
__device__ __forceinline__ float numpy_row_sum(const float* v, int n) {
  if (n < 8) {
    float total = 0.f;
    for (int i = 0; i < n; ++i) total = __fadd_rn(total, v[i]);
    return total;
  }
  if constexpr (kDepth == 0) {
    return numpy_block_sum(v, n);
  } else {
    if (n <= 128) return numpy_block_sum(v, n);
    int half = n / 2;
    half -= half % 8;
    const float left = numpy_row_sum<kDepth - 1>(v, half);
    const float right = numpy_row_sum<kDepth - 1>(v + half, n - half);
    return __fadd_rn(left, right);
  }
}

}  // namespace cg
