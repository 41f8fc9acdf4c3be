// Policy/value heads, legal-action masking and inverse-CDF sampling for a wave of decisions.
//
// Reference: cardgym/games/plump/model.py:204-217 (bid Linear, 52 card logits
// h . (rank[r] + suit[s]) + bias, value MLP), cardgym/rl/selfplay.py:486-567
// (launch_policies groups decisions by head and samples on the host),
// cardgym/rl/ppo.py:75-94 (masked_probabilities, sample_rows).
//
// Sampling semantics follow the reference exactly: illegal logits -> -inf, shift by
// the legal max, exp, illegal -> 0, divide by the sum; draw = #{k : cumsum_k < u},
// clamped to the last legal index, an illegal draw replaced by the last legal index.
// exp is evaluated in float64 and rounded once (a correctly rounded float32 exp);
// the reference's numpy float32 exp carries up to ~2.4 ulp of error, so
// probabilities agree to a few ulp and draws agree except within a few ulp of a
// CDF step.
#include "common.cuh"

namespace cg {

constexpr int kMaxSampleWidth = 256;

// One warp samples one row. probs_s: per-warp shared buffer of kMaxSampleWidth floats.
__device__ void warp_sample(const float* logits, const uint8_t* mask, int width, double u, float* probs_s,
                            float* probs_out, int64_t* action_out) {
  const int lane = threadIdx.x & 31;
  float peak = -INFINITY;
  int last_legal = -1;
  for (int j = lane; j < width; j += 32) {
    if (mask[j]) {
      peak = fmaxf(peak, logits[j]);
      last_legal = j;
    }
  }
  peak = warp_max(peak);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last_legal = max(last_legal, __shfl_xor_sync(0xffffffffu, last_legal, o));
  float total = 0.f;
  for (int j = lane; j < width; j += 32) {
    float e = 0.f;
    if (mask[j]) e = static_cast<float>(exp(static_cast<double>(logits[j] - peak)));
    probs_s[j] = e;
    total += e;
  }
  total = warp_sum(total);
  __syncwarp();
  for (int j = lane; j < width; j += 32) {
    const float p = probs_s[j] / total;
    probs_s[j] = p;
    if (probs_out) probs_out[j] = p;
  }
  __syncwarp();
  if (lane == 0) {
    float cdf = 0.f;
    int below = 0;
    for (int j = 0; j < width; ++j) {
      cdf += probs_s[j];
      below += static_cast<double>(cdf) < u ? 1 : 0;
    }
    int drawn = last_legal < 0 ? 0 : min(below, last_legal);
    if (last_legal >= 0 && !mask[drawn]) drawn = last_legal;
    *action_out = drawn;
  }
  __syncwarp();
}

__global__ void masked_sample_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ mask,
                                     const double* __restrict__ uniforms, int64_t rows, int width, float* probs_out,
                                     int64_t* actions_out) {
  __shared__ float probs_s[4][kMaxSampleWidth];
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= rows) return;
  warp_sample(logits + row * width, mask + row * width, width, uniforms[row], probs_s[threadIdx.x >> 5],
              probs_out ? probs_out + row * width : nullptr, actions_out + row);
}

// One CTA (4 warps) per decision.
__global__ void __launch_bounds__(128) decide_kernel(cg_heads_desc desc, const float* __restrict__ blob,
                                                      const float* __restrict__ hidden,
                                                      const int64_t* __restrict__ hidden_rows, int64_t decisions,
                                                      const int32_t* __restrict__ head_of,
                                                      const uint8_t* __restrict__ legal,
                                                      const double* __restrict__ uniforms, float* logits_out,
                                                      float* probs_out, int64_t* actions_out, float* values_out) {
  extern __shared__ float sm[];
  const int d = desc.d_model, W = desc.max_width;
  float* h = sm;                // [d]
  float* hid = h + d;           // [d] value MLP hidden
  float* logit_s = hid + d;     // [W]
  float* probs_s = logit_s + W; // [W]
  const int64_t i = blockIdx.x;
  if (i >= decisions) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t src = hidden_rows ? hidden_rows[i] : i;
  for (int k = threadIdx.x; k < d; k += blockDim.x) h[k] = hidden[src * d + k];
  __syncthreads();
  const int head = head_of ? head_of[i] : 0;
  const bool head_ok = head >= 0 && head < desc.n_policy;
  if (!head_ok && threadIdx.x == 0) raise_fault(0x300);
  const int A = head_ok ? desc.width[head] : 0;
  const float* Wh = blob + (head_ok ? desc.weight_offset[head] : 0);
  const float* bh = blob + (head_ok ? desc.bias_offset[head] : 0);
  for (int a = warp; a < W; a += 4) {
    float acc = 0.f;
    if (a < A) {
      for (int k = lane; k < d; k += 32) acc = fmaf(Wh[static_cast<int64_t>(a) * d + k], h[k], acc);
      acc = warp_sum(acc) + bh[a];
    }
    if (lane == 0) {
      logit_s[a] = a < A ? acc : -INFINITY;
      if (logits_out) logits_out[i * W + a] = a < A ? acc : 0.f;
    }
  }
  __syncthreads();
  if (warp == 0) {
    // Entries past the head's width are never legal.
    const uint8_t* mask = legal + i * W;
    __shared__ uint8_t mask_s[kMaxSampleWidth];
    for (int a = lane; a < W; a += 32) mask_s[a] = a < A ? mask[a] : 0;
    __syncwarp();
    warp_sample(logit_s, mask_s, W, uniforms[i], probs_s, probs_out ? probs_out + i * W : nullptr, actions_out + i);
  }
  if (desc.value_outputs > 0 && values_out) {
    const float* W1 = blob + desc.value_w1;
    const float* b1 = blob + desc.value_b1;
    for (int o = warp; o < d; o += 4) {
      float acc = 0.f;
      for (int k = lane; k < d; k += 32) acc = fmaf(W1[static_cast<int64_t>(o) * d + k], h[k], acc);
      acc = warp_sum(acc) + b1[o];
      if (lane == 0) hid[o] = gelu_erf(acc);
    }
    __syncthreads();
    const float* W2 = blob + desc.value_w2;
    const float* b2 = blob + desc.value_b2;
    for (int o = warp; o < desc.value_outputs; o += 4) {
      float acc = 0.f;
      for (int k = lane; k < d; k += 32) acc = fmaf(W2[static_cast<int64_t>(o) * d + k], hid[k], acc);
      acc = warp_sum(acc) + b2[o];
      if (lane == 0) values_out[i * desc.value_outputs + o] = acc;
    }
  }
}

}  // namespace cg

extern "C" int cg_masked_sample(const float* logits, const uint8_t* mask, const double* uniforms, int64_t rows,
                                int width, float* probs_out, int64_t* actions_out, void* stream) {
  using namespace cg;
  CG_REQUIRE(rows >= 0 && width > 0 && width <= kMaxSampleWidth, "cg_masked_sample: width must be 1..%d",
             kMaxSampleWidth);
  if (rows == 0) return CG_OK;
  CG_REQUIRE(logits && mask && uniforms && actions_out, "cg_masked_sample: NULL pointer");
  masked_sample_kernel<<<static_cast<unsigned>((rows + 3) / 4), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, mask, uniforms, rows, width, probs_out, actions_out);
  return check_launch("masked_sample_kernel");
}

extern "C" int cg_plump_decide(const cg_heads_desc* desc, const float* heads_blob, const float* hidden,
                               const int64_t* hidden_rows, int64_t decisions, const int32_t* head_of,
                               const uint8_t* legal, const double* uniforms, float* logits_out, float* probs_out,
                               int64_t* actions_out, float* values_out, void* stream) {
  using namespace cg;
  CG_REQUIRE(desc, "cg_plump_decide: NULL desc");
  CG_REQUIRE(desc->d_model > 0 && desc->n_policy >= 1 && desc->n_policy <= 8, "cg_plump_decide: bad desc");
  CG_REQUIRE(desc->max_width > 0 && desc->max_width <= kMaxSampleWidth, "cg_plump_decide: max_width must be 1..%d",
             kMaxSampleWidth);
  for (int h = 0; h < desc->n_policy; ++h)
    CG_REQUIRE(desc->width[h] > 0 && desc->width[h] <= desc->max_width, "cg_plump_decide: head %d width", h);
  if (decisions == 0) return CG_OK;
  CG_REQUIRE(heads_blob && hidden && legal && uniforms && actions_out, "cg_plump_decide: NULL pointer");
  CG_REQUIRE(decisions <= 0x7fffffff, "cg_plump_decide: too many decisions");
  const size_t smem = (2 * desc->d_model + 2 * desc->max_width) * sizeof(float);
  CG_REQUIRE(smem <= 48 * 1024, "cg_plump_decide: d_model too large");
  decide_kernel<<<static_cast<unsigned>(decisions), 128, smem, static_cast<cudaStream_t>(stream)>>>(
      *desc, heads_blob, hidden, hidden_rows, decisions, head_of, legal, uniforms, logits_out, probs_out, actions_out,
      values_out);
  return check_launch("decide_kernel");
}
