/* numpy's float32 exp and last-axis sum, restated in C -- TEST INFRASTRUCTURE ONLY.
 *
 * The reference samples decisions with numpy float32 (cardgym/rl/ppo.py:75-94): np.exp of
 * the shifted logits and weights.sum(axis=-1). On x86-64 hosts with AVX2+FMA3 or AVX-512F,
 * numpy 2.3 evaluates float32 exp with the SIMD routine of
 * numpy/_core/src/umath/loops_exponent_log.dispatch.c.src: k = rint(x log2 e), a two-step
 * Cody-Waite reduction r = x - k ln2, a degree-5 / degree-2 rational approximation
 * P(r)/Q(r), and the result scaled by 2^k (x >= 88.7228 -> inf, x <= -103.972 -> 0).
 * Its last-axis float32 add-reduction is pairwise_sum
 * (numpy/_core/src/umath/loops_utils.h.src) from the identity 0.
 *
 * The device kernels restate the same two functions (card_playing_gym_b200/csrc/
 * numpy_math.cuh). This C copy lets CPU tests pin the restatement against np.exp and
 * np.sum themselves, so that a GPU test that compares the kernels with numpy tests the
 * kernels rather than the restatement.
 */
#include <math.h>
#include <stdint.h>

static const float kLog2e = 0x1.715476p+0f;
static const float kLn2Hi = -6.93145752e-1f;
static const float kLn2Lo = -1.42860677e-6f;
static const float kP[6] = {9.999999999980870924916e-01f, 7.257664613233124478488e-01f,
                            2.473615434895520810817e-01f, 5.114512081637298353406e-02f,
                            6.757896990527504603057e-03f, 5.082762800157070e-04f};
static const float kQ1 = -2.742335390411667452936e-01f;
static const float kQ2 = 2.159509375685829852307e-02f;

float oracle_numpy_expf(float x) {
  if (x != x) return x;
  if (x >= 88.72283935546875f) return INFINITY;
  if (x <= -103.97208404541015625f) return 0.0f;
  volatile float scaled = x * kLog2e; /* one float32 rounding, never fused */
  const float k = rintf(scaled);
  float r = fmaf(k, kLn2Hi, x);
  r = fmaf(k, kLn2Lo, r);
  float num = fmaf(kP[5], r, kP[4]);
  num = fmaf(num, r, kP[3]);
  num = fmaf(num, r, kP[2]);
  num = fmaf(num, r, kP[1]);
  num = fmaf(num, r, kP[0]);
  float den = fmaf(kQ2, r, kQ1);
  den = fmaf(den, r, 1.0f);
  volatile float quotient = num / den;
  return ldexpf(quotient, (int)k);
}

void oracle_numpy_expf_array(const float* x, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = oracle_numpy_expf(x[i]);
}

static float pairwise(const float* a, int64_t n) {
  if (n < 8) {
    float res = 0.0f;
    for (int64_t i = 0; i < n; ++i) res += a[i];
    return res;
  }
  if (n <= 128) {
    float r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    int64_t i = 8;
    for (; i < n - (n % 8); i += 8)
      for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
    return res;
  }
  int64_t half = n / 2;
  half -= half % 8;
  return pairwise(a, half) + pairwise(a + half, n - half);
}

/* Row sums of a C-contiguous [rows, width] float32 matrix, numpy's order. */
void oracle_numpy_row_sums(const float* a, int64_t rows, int64_t width, float* out) {
  for (int64_t r = 0; r < rows; ++r) out[r] = 0.0f + pairwise(a + r * width, width);
}
