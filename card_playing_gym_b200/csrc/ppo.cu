// PPO advantage and loss step: segmented GAE, batch-global normalisation sums, the fused
// per-head PPO objective with its gradient w.r.t. the logits, and the dense value loss.
//
// Reference: cardgym/rl/ppo.py (ppo_terms 28-72, center_zero_sum 97-108,
// gae_advantages 121-144, weighted_mean_std 147-153) and cardgym/rl/trainer.py
// (_gae 634-649, _policy_loss 733-802, _value_loss 822-850). Totals reduce
// deterministically: fixed-size grids write per-block float64 partials to the
// workspace and one block sums them in order.
#include "common.cuh"

namespace cg {

constexpr int kReduceBlocks = 512;  // fixed partial count: the same order on every call
constexpr int kObjectiveBlocks = 2048;  // the objective's partial count (8 rows in flight per block)
constexpr int kTerms = 8;

// ---- GAE -----------------------------------------------------------------------------
// Thread per (game, seat): running = (next - V[s]) + lambda * running, last state first;
// written where the row's acting seat is this seat. Rounding steps match numpy's.
__global__ void gae_kernel(const double* __restrict__ values, int players, const int32_t* __restrict__ seats,
                           const int64_t* __restrict__ starts, int64_t games, const double* __restrict__ returns,
                           double lambda, double* __restrict__ out) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i >= games * players) return;
  const int64_t game = i / players;
  const int seat = static_cast<int>(i % players);
  const int64_t lo = starts[game], hi = starts[game + 1];
  double next = returns[game * players + seat];
  double running = 0.0;
  for (int64_t row = hi - 1; row >= lo; --row) {
    const double v = values[row * players + seat];
    running = __dadd_rn(__dsub_rn(next, v), __dmul_rn(lambda, running));
    if (seats[row] == seat) out[row] = running;
    next = v;
  }
}

// ---- weighted sums ---------------------------------------------------------------------
// mean = sum w x / sum w from a first pass's sums (0 without weight), as mean_std_from_sums.
__device__ __forceinline__ double mean_from_sums(const double* first) {
  return first[0] > 0 ? first[1] / first[0] : 0.0;
}

// shift_from: when non-null, the shift is the mean of a first pass's sums, read on the device.
__global__ void weighted_sums_kernel(const double* __restrict__ x, const double* __restrict__ w, int64_t n,
                                     double shift, const double* __restrict__ shift_from, double* partial) {
  __shared__ double s[3][256];
  if (shift_from) shift = mean_from_sums(shift_from);
  double a = 0, b = 0, c = 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const double dx = x[i] - shift;
    a += w[i];
    b += w[i] * dx;
    c += w[i] * dx * dx;
  }
  s[0][threadIdx.x] = a;
  s[1][threadIdx.x] = b;
  s[2][threadIdx.x] = c;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o)
      for (int k = 0; k < 3; ++k) s[k][threadIdx.x] += s[k][threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x < 3) partial[blockIdx.x * 3 + threadIdx.x] = s[threadIdx.x][0];
}

// Sums `count` partial rows of `width` doubles into out[width]: warp k takes column k, lane l
// the partials l, l + 32, ... in order, then a fixed butterfly; the same order on every call.
__global__ void sum_partials_kernel(const double* partial, int count, int width, double* out) {
  const int lane = threadIdx.x & 31;
  for (int k = threadIdx.x >> 5; k < width; k += blockDim.x >> 5) {
    double total = 0;
    for (int b = lane; b < count; b += 32) total += partial[b * width + k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (lane == 0) out[k] = total;
  }
}

__global__ void normalize_kernel(double* x, int64_t n, double mean, double std) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = (x[i] - mean) / std;
}

// The same with mean and std from the two passes' sums on the device (ppo.py:147-153:
// mean = sum w x / sum w, std = sqrt(max(sum w (x - mean)^2 / sum w, 1e-12)); (0, 1) without weight).
__global__ void normalize_from_sums_kernel(double* x, int64_t n, const double* __restrict__ first,
                                           const double* __restrict__ second) {
  const double total = first[0];
  const double mean = total > 0 ? first[1] / total : 0.0;
  const double std = total > 0 ? sqrt(fmax(second[2] / total, 1e-12)) : 1.0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = (x[i] - mean) / std;
}

// ---- fused PPO objective ---------------------------------------------------------------
constexpr int kPpoMaxWidth = 256;

// kPer: logits per lane (width <= 32 * kPer).
template <int kPer>
__global__ void __launch_bounds__(256) ppo_objective_kernel(
    const float* __restrict__ logits, const float* __restrict__ old_probs, int64_t rows, int width, int64_t stride,
    const int64_t* __restrict__ actions, const float* __restrict__ advantages, const float* __restrict__ weights,
    float clip, float alpha, float* dlogits, float* row_terms, double* partial) {
  __shared__ double s[8][kTerms];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double acc[kTerms] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t step = static_cast<int64_t>(gridDim.x) * 8;
  // The next row's inputs load while this row is computed.
  float nz[kPer], no[kPer];
  int64_t na = 0;
  float nadv = 0.f, nw = 0.f;
  auto fetch = [&](int64_t r) {
    if (r >= rows) return;
    const float* z = logits + r * stride;
    const float* old = old_probs + r * stride;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int j = lane + 32 * k;
      nz[k] = j < width ? z[j] : 0.f;
      no[k] = j < width ? old[j] : 0.f;
    }
    na = actions[r];
    nadv = advantages[r];
    nw = weights[r];
  };
  fetch(static_cast<int64_t>(blockIdx.x) * 8 + warp);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + warp; row < rows; row += step) {
    float zl[kPer], ol[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      zl[k] = nz[k];
      ol[k] = no[k];
    }
    const int64_t a = na;
    const float adv = nadv, w = nw;
    fetch(row + step);
    float peak = -INFINITY;
    int count = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      if (ol[k] > 0.f) {
        peak = fmaxf(peak, zl[k]);
        ++count;
      }
    }
    peak = warp_max(peak);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) count += __shfl_xor_sync(0xffffffffu, count, o);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      if (ol[k] > 0.f) sum += expf(zl[k] - peak);
    sum = warp_sum(sum);
    const float lse = peak + logf(sum);
    float lp_a = 0.f, old_log_a = 0.f;
    float entropy = 0.f, kl = 0.f;
    float lp[kPer], p[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int j = lane + 32 * k;
      const bool legal = ol[k] > 0.f;
      lp[k] = legal ? zl[k] - lse : 0.f;
      p[k] = legal ? expf(lp[k]) : 0.f;
      const float old_log = logf(fmaxf(ol[k], 1e-12f));
      if (j == a) {
        lp_a = lp[k];
        old_log_a = old_log;
      }
      if (legal) {
        entropy -= p[k] * lp[k];
        kl += ol[k] * (old_log - lp[k]);
      }
    }
    lp_a = warp_sum(lp_a);  // exactly one lane holds the action's value
    old_log_a = warp_sum(old_log_a);
    entropy = warp_sum(entropy);
    kl = warp_sum(kl);
    const float ratio = expf(lp_a - old_log_a);
    const float clipped_ratio = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip);
    const float unclipped = ratio * adv, clipped = clipped_ratio * adv;
    const float loss = -fminf(unclipped, clipped);
    // d(-min(rA, clip(r)A))/dr with torch's tie and clamp-boundary conventions.
    const bool inside = ratio >= 1.f - clip && ratio <= 1.f + clip;
    const float d_ratio = unclipped < clipped ? -adv : (unclipped > clipped ? (inside ? -adv : 0.f) : -adv);
    const bool eligible = count > 1;
    const float norm_scale = eligible ? 1.f / logf(static_cast<float>(count < 2 ? 2 : count)) : 0.f;
    const float normalized = eligible ? entropy * norm_scale : 0.f;
    const bool is_clipped = fabsf(ratio - 1.f) > clip;
    if (dlogits) {
      const float g_action = w * d_ratio * ratio;
      const float g_entropy = -alpha * w * norm_scale;
#pragma unroll
      for (int k = 0; k < kPer; ++k) {
        const int j = lane + 32 * k;
        if (j >= width) continue;
        float g = 0.f;
        if (ol[k] > 0.f) {
          g = g_action * ((j == a ? 1.f : 0.f) - p[k]);
          g += g_entropy * (-p[k] * (lp[k] + entropy));
        }
        dlogits[row * width + j] = g;
      }
    }
    if (row_terms && lane == 0) {
      float* t = row_terms + row * kTerms;
      t[0] = loss;
      t[1] = kl;
      t[2] = entropy;
      t[3] = normalized;
      t[4] = eligible ? 1.f : 0.f;
      t[5] = ratio;
      t[6] = is_clipped ? 1.f : 0.f;
      t[7] = lp_a;
    }
    const double wd = w;
    acc[0] += wd * loss;
    acc[1] += wd;
    acc[2] += wd * entropy;
    acc[3] += wd * (eligible ? 1.0 : 0.0) * normalized;
    acc[4] += eligible ? wd : 0.0;
    acc[5] += is_clipped ? wd : 0.0;
    acc[6] += wd * kl;
    acc[7] += wd * loss - static_cast<double>(alpha) * wd * (eligible ? 1.0 : 0.0) * normalized;
  }
  if (lane == 0)
    for (int k = 0; k < kTerms; ++k) s[warp][k] = acc[k];
  __syncthreads();
  if (threadIdx.x < kTerms) {
    double total = 0;
    for (int w = 0; w < 8; ++w) total += s[w][threadIdx.x];
    partial[blockIdx.x * kTerms + threadIdx.x] = total;
  }
}

// Rows of at most 64 legal-masked logits (width % 4 == 0, 16-byte aligned rows): eight lanes
// per row, four rows per warp. Lane l of a row group holds logits 4l..4l+3 and 32+4l..32+4l+3
// (float4 loads and stores); the row's reductions are three butterfly steps inside the group.
// The same arithmetic as ppo_objective_kernel; only the order of the per-row sums differs.
__device__ __forceinline__ float group8_sum(float v) {
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) ppo_objective_narrow_kernel(
    const float* __restrict__ logits, const float* __restrict__ old_probs, int64_t rows, int width, int64_t stride,
    const int64_t* __restrict__ actions, const float* __restrict__ advantages, const float* __restrict__ weights,
    float clip, float alpha, float* dlogits, float* row_terms, double* partial) {
  __shared__ double s[8][kTerms];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int grp = lane >> 3, l = lane & 7;
  double acc[kTerms] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int64_t step = static_cast<int64_t>(gridDim.x) * 32;
  float4 nz[2], no[2];
  int64_t na = 0;
  float nadv = 0.f, nw = 0.f;
  auto fetch = [&](int64_t r) {
    if (r >= rows) return;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 4 * l + 32 * h;
      nz[h] = j < width ? *reinterpret_cast<const float4*>(logits + r * stride + j) : make_float4(0.f, 0.f, 0.f, 0.f);
      no[h] = j < width ? *reinterpret_cast<const float4*>(old_probs + r * stride + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    na = actions[r];
    nadv = advantages[r];
    nw = weights[r];
  };
  // Every group of a warp runs the same iterations, so the shuffles stay converged.
  const int64_t warp_first = (static_cast<int64_t>(blockIdx.x) * 8 + warp) * 4;
  fetch(warp_first + grp);
  for (int64_t base = warp_first; base < rows; base += step) {
    const int64_t row = base + grp;
    const bool live = row < rows;
    float zl[8], ol[8];
    zl[0] = nz[0].x, zl[1] = nz[0].y, zl[2] = nz[0].z, zl[3] = nz[0].w;
    zl[4] = nz[1].x, zl[5] = nz[1].y, zl[6] = nz[1].z, zl[7] = nz[1].w;
    ol[0] = no[0].x, ol[1] = no[0].y, ol[2] = no[0].z, ol[3] = no[0].w;
    ol[4] = no[1].x, ol[5] = no[1].y, ol[6] = no[1].z, ol[7] = no[1].w;
    if (!live) {
#pragma unroll
      for (int k = 0; k < 8; ++k) ol[k] = 0.f;  // nothing legal: the padding row contributes nothing
    }
    const int64_t a = na;
    const float adv = live ? nadv : 0.f, w = live ? nw : 0.f;
    fetch(row + step);
    float peak = -INFINITY;
    float count = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (ol[k] > 0.f) {
        peak = fmaxf(peak, zl[k]);
        count += 1.f;
      }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, o));
    count = group8_sum(count);
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (ol[k] > 0.f) sum += expf(zl[k] - peak);
    sum = group8_sum(sum);
    const float lse = peak + logf(sum);
    float lp_a = 0.f, old_log_a = 0.f, entropy = 0.f, kl = 0.f;
    float lp[8], p[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = 4 * l + 32 * (k >> 2) + (k & 3);
      const bool legal = ol[k] > 0.f;
      lp[k] = legal ? zl[k] - lse : 0.f;
      p[k] = legal ? expf(lp[k]) : 0.f;
      const float old_log = logf(fmaxf(ol[k], 1e-12f));
      if (j == a) {
        lp_a = lp[k];
        old_log_a = old_log;
      }
      if (legal) {
        entropy -= p[k] * lp[k];
        kl += ol[k] * (old_log - lp[k]);
      }
    }
    lp_a = group8_sum(lp_a);
    old_log_a = group8_sum(old_log_a);
    entropy = group8_sum(entropy);
    kl = group8_sum(kl);
    const float ratio = expf(lp_a - old_log_a);
    const float clipped_ratio = fminf(fmaxf(ratio, 1.f - clip), 1.f + clip);
    const float unclipped = ratio * adv, clipped = clipped_ratio * adv;
    const float loss = -fminf(unclipped, clipped);
    const bool inside = ratio >= 1.f - clip && ratio <= 1.f + clip;
    const float d_ratio = unclipped < clipped ? -adv : (unclipped > clipped ? (inside ? -adv : 0.f) : -adv);
    const int icount = static_cast<int>(count);
    const bool eligible = icount > 1;
    const float norm_scale = eligible ? 1.f / logf(static_cast<float>(icount < 2 ? 2 : icount)) : 0.f;
    const float normalized = eligible ? entropy * norm_scale : 0.f;
    const bool is_clipped = fabsf(ratio - 1.f) > clip;
    if (dlogits && live) {
      const float g_action = w * d_ratio * ratio;
      const float g_entropy = -alpha * w * norm_scale;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j0 = 4 * l + 32 * h;
        if (j0 >= width) continue;
        float g[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = 4 * h + e;
          g[e] = 0.f;
          if (ol[k] > 0.f) {
            g[e] = g_action * ((j0 + e == a ? 1.f : 0.f) - p[k]);
            g[e] += g_entropy * (-p[k] * (lp[k] + entropy));
          }
        }
        *reinterpret_cast<float4*>(dlogits + row * width + j0) = make_float4(g[0], g[1], g[2], g[3]);
      }
    }
    if (row_terms && live && l == 0) {
      float* t = row_terms + row * kTerms;
      t[0] = loss;
      t[1] = kl;
      t[2] = entropy;
      t[3] = normalized;
      t[4] = eligible ? 1.f : 0.f;
      t[5] = ratio;
      t[6] = is_clipped ? 1.f : 0.f;
      t[7] = lp_a;
    }
    if (l == 0 && live) {
      const double wd = w;
      acc[0] += wd * loss;
      acc[1] += wd;
      acc[2] += wd * entropy;
      acc[3] += wd * (eligible ? 1.0 : 0.0) * normalized;
      acc[4] += eligible ? wd : 0.0;
      acc[5] += is_clipped ? wd : 0.0;
      acc[6] += wd * kl;
      acc[7] += wd * loss - static_cast<double>(alpha) * wd * (eligible ? 1.0 : 0.0) * normalized;
    }
  }
  // The four group leaders' sums in group order, then the warps in order.
#pragma unroll
  for (int k = 0; k < kTerms; ++k) {
    const double v = acc[k];
    const double v8 = __shfl_down_sync(0xffffffffu, v, 8);
    const double v16 = __shfl_down_sync(0xffffffffu, v, 16);
    const double v24 = __shfl_down_sync(0xffffffffu, v, 24);
    acc[k] = ((v + v8) + v16) + v24;
  }
  if (lane == 0)
    for (int k = 0; k < kTerms; ++k) s[warp][k] = acc[k];
  __syncthreads();
  if (threadIdx.x < kTerms) {
    double total = 0;
    for (int w = 0; w < 8; ++w) total += s[w][threadIdx.x];
    partial[blockIdx.x * kTerms + threadIdx.x] = total;
  }
}

// ---- value loss ---------------------------------------------------------------------------
constexpr int kValueMaxPlayers = 16;

__global__ void value_loss_kernel(const float* __restrict__ pred, const float* __restrict__ targets,
                                  const int32_t* __restrict__ players, const float* __restrict__ weights, int64_t rows,
                                  int P, float scale, float* grad, double* partial) {
  __shared__ double s[4][256];
  double acc[4] = {0, 0, 0, 0};
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int n = players[r];
    const float w = weights[r];
    const float nf = static_cast<float>(n);
    float mean = 0.f;
    for (int j = 0; j < P; ++j) mean += j < n ? pred[r * P + j] : 0.f;
    mean = mean / nf;
    float sq_err = 0.f, sq_raw = 0.f, sq_tgt = 0.f, gsum = 0.f;
    float g[kValueMaxPlayers];
    for (int j = 0; j < P; ++j) {
      const bool active = j < n;
      const float centered = active ? (pred[r * P + j] - mean) : 0.f;
      const float tgt = targets[r * P + j];
      const float raw = centered - tgt;
      const float err = raw / scale;
      if (active) {
        sq_err += err * err;
        sq_raw += raw * raw;
        sq_tgt += tgt * tgt;
      }
      g[j] = active ? (w / nf) * err / scale : 0.f;
      gsum += g[j];
    }
    if (grad)
      for (int j = 0; j < P; ++j) grad[r * P + j] = j < n ? g[j] - gsum / nf : 0.f;
    acc[0] += 0.5 * w * sq_err / nf;
    acc[1] += static_cast<double>(w / nf) * sq_raw;
    acc[2] += static_cast<double>(w / nf) * sq_tgt;
    acc[3] += w;
  }
  for (int k = 0; k < 4; ++k) s[k][threadIdx.x] = acc[k];
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o)
      for (int k = 0; k < 4; ++k) s[k][threadIdx.x] += s[k][threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x < 4) partial[blockIdx.x * 4 + threadIdx.x] = s[threadIdx.x][0];
}

int reduce_blocks(int64_t items, int per_block) {
  int64_t b = (items + per_block - 1) / per_block;
  if (b < 1) b = 1;
  return static_cast<int>(b > kReduceBlocks ? kReduceBlocks : b);
}

}  // namespace cg

extern "C" int cg_gae_segments(const double* values, int players, const int32_t* seats, const int64_t* starts,
                               int64_t games, const double* returns, double gae_lambda, double* advantages_out,
                               void* stream) {
  using namespace cg;
  CG_REQUIRE(players > 0 && games >= 0, "cg_gae_segments: bad shape");
  if (games == 0) return CG_OK;
  CG_REQUIRE(values && seats && starts && returns && advantages_out, "cg_gae_segments: NULL pointer");
  const int64_t threads = games * players;
  gae_kernel<<<static_cast<unsigned>((threads + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      values, players, seats, starts, games, returns, gae_lambda, advantages_out);
  return check_launch("gae_kernel");
}

extern "C" int64_t cg_weighted_sums_workspace_bytes(int64_t) { return cg::kReduceBlocks * 3 * sizeof(double); }

extern "C" int cg_weighted_sums(const double* values, const double* weights, int64_t n, double shift, double* out3,
                                void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace cg;
  CG_REQUIRE(n >= 0 && out3 && workspace, "cg_weighted_sums: bad arguments");
  CG_REQUIRE(n == 0 || (values && weights), "cg_weighted_sums: NULL input");
  const int blocks = reduce_blocks(n, 256);
  if (workspace_bytes < static_cast<int64_t>(blocks) * 3 * 8)
    return set_error(CG_ERR_WORKSPACE, "cg_weighted_sums: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  weighted_sums_kernel<<<blocks, 256, 0, s>>>(values, weights, n, shift, nullptr, partial);
  int rc = check_launch("weighted_sums_kernel");
  if (rc) return rc;
  sum_partials_kernel<<<1, 3 * 32, 0, s>>>(partial, blocks, 3, out3);
  return check_launch("sum_partials_kernel");
}

extern "C" int cg_weighted_sums_shifted(const double* values, const double* weights, int64_t n,
                                        const double* shift_sums3, double* out3, void* workspace,
                                        int64_t workspace_bytes, void* stream) {
  using namespace cg;
  CG_REQUIRE(n >= 0 && out3 && workspace && shift_sums3, "cg_weighted_sums_shifted: bad arguments");
  CG_REQUIRE(n == 0 || (values && weights), "cg_weighted_sums_shifted: NULL input");
  const int blocks = reduce_blocks(n, 256);
  if (workspace_bytes < static_cast<int64_t>(blocks) * 3 * 8)
    return set_error(CG_ERR_WORKSPACE, "cg_weighted_sums_shifted: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  weighted_sums_kernel<<<blocks, 256, 0, s>>>(values, weights, n, 0.0, shift_sums3, partial);
  int rc = check_launch("weighted_sums_kernel");
  if (rc) return rc;
  sum_partials_kernel<<<1, 3 * 32, 0, s>>>(partial, blocks, 3, out3);
  return check_launch("sum_partials_kernel");
}

extern "C" int cg_normalize_from_sums(double* values, int64_t n, const double* first3, const double* second3,
                                      void* stream) {
  using namespace cg;
  CG_REQUIRE(n >= 0 && first3 && second3, "cg_normalize_from_sums: bad arguments");
  if (n == 0) return CG_OK;
  CG_REQUIRE(values, "cg_normalize_from_sums: NULL values");
  normalize_from_sums_kernel<<<reduce_blocks(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(values, n, first3,
                                                                                                  second3);
  return check_launch("normalize_from_sums_kernel");
}

extern "C" int cg_normalize(double* values, int64_t n, double mean, double std, void* stream) {
  using namespace cg;
  CG_REQUIRE(n >= 0 && std > 0, "cg_normalize: bad arguments");
  if (n == 0) return CG_OK;
  CG_REQUIRE(values, "cg_normalize: NULL values");
  normalize_kernel<<<reduce_blocks(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(values, n, mean, std);
  return check_launch("normalize_kernel");
}

extern "C" int64_t cg_ppo_objective_workspace_bytes(int64_t) { return cg::kObjectiveBlocks * cg::kTerms * sizeof(double); }

namespace cg {
// Blocks of the objective that are resident at once. The grid is one such wave: every warp keeps
// its next rows' loads in flight through the grid-stride loop, and a grid of several waves
// leaves its last wave part-empty (measured: the 262,144-row step 0.180 ms against 0.189 ms
// with 2,048 blocks).
static int resident_objective_blocks() {
  static int per_sm = 0;
  if (!per_sm && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ppo_objective_narrow_kernel, 256, 0) !=
                      cudaSuccess ||
                  per_sm < 1))
    per_sm = 1;
  return per_sm * sm_count();
}
}  // namespace cg

extern "C" int cg_ppo_objective(const float* logits, const float* old_probs, int64_t rows, int width, int64_t stride,
                                const int64_t* actions, const float* advantages, const float* weights, float clip_ratio,
                                float alpha, float* dlogits, float* row_terms, double* totals, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  using namespace cg;
  CG_REQUIRE(rows >= 0 && width > 0 && width <= kPpoMaxWidth, "cg_ppo_objective: width must be 1..%d", kPpoMaxWidth);
  CG_REQUIRE(stride >= width, "cg_ppo_objective: stride < width");
  if (rows == 0) return CG_OK;
  CG_REQUIRE(logits && old_probs && actions && advantages && weights, "cg_ppo_objective: NULL input");
  CG_REQUIRE(!totals || workspace, "cg_ppo_objective: totals need a workspace");
  const int64_t cap = std::min<int64_t>(kObjectiveBlocks, resident_objective_blocks());
  const int64_t want = (rows + 7) / 8;
  const int blocks = static_cast<int>(want < cap ? want : cap);
  if (totals && workspace_bytes < static_cast<int64_t>(blocks) * kTerms * 8)
    return set_error(CG_ERR_WORKSPACE, "cg_ppo_objective: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  // Without totals the partials still need a home: the kernel writes them unconditionally.
  if (!partial) return set_error(CG_ERR_WORKSPACE, "cg_ppo_objective: workspace required");
  const bool narrow = width <= 64 && width % 4 == 0 && stride % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(logits) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(old_probs) & 15) == 0 &&
                      (!dlogits || (reinterpret_cast<uintptr_t>(dlogits) & 15) == 0);
  if (narrow)
    ppo_objective_narrow_kernel<<<blocks, 256, 0, s>>>(logits, old_probs, rows, width, stride, actions, advantages,
                                                       weights, clip_ratio, alpha, dlogits, row_terms, partial);
  else if (width <= 64)
    ppo_objective_kernel<2><<<blocks, 256, 0, s>>>(logits, old_probs, rows, width, stride, actions, advantages,
                                                   weights, clip_ratio, alpha, dlogits, row_terms, partial);
  else
    ppo_objective_kernel<kPpoMaxWidth / 32><<<blocks, 256, 0, s>>>(logits, old_probs, rows, width, stride, actions,
                                                                   advantages, weights, clip_ratio, alpha, dlogits,
                                                                   row_terms, partial);
  int rc = check_launch("ppo_objective_kernel");
  if (rc || !totals) return rc;
  sum_partials_kernel<<<1, kTerms * 32, 0, s>>>(partial, blocks, kTerms, totals);
  return check_launch("sum_partials_kernel");
}

extern "C" int64_t cg_value_loss_workspace_bytes(int64_t) { return cg::kReduceBlocks * 4 * sizeof(double); }

extern "C" int cg_value_loss(const float* prediction, const float* targets, const int32_t* players,
                             const float* weights, int64_t rows, int players_max, float reward_scale, float* grad,
                             double* totals, void* workspace, int64_t workspace_bytes, void* stream) {
  using namespace cg;
  CG_REQUIRE(rows >= 0 && players_max > 0 && players_max <= kValueMaxPlayers, "cg_value_loss: players_max 1..%d",
             kValueMaxPlayers);
  CG_REQUIRE(reward_scale > 0, "cg_value_loss: reward_scale must be positive");
  if (rows == 0) return CG_OK;
  CG_REQUIRE(prediction && targets && players && weights && workspace, "cg_value_loss: NULL pointer");
  const int blocks = reduce_blocks(rows, 256);
  if (workspace_bytes < static_cast<int64_t>(blocks) * 4 * 8)
    return set_error(CG_ERR_WORKSPACE, "cg_value_loss: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  value_loss_kernel<<<blocks, 256, 0, s>>>(prediction, targets, players, weights, rows, players_max, reward_scale,
                                           grad, partial);
  int rc = check_launch("value_loss_kernel");
  if (rc || !totals) return rc;
  sum_partials_kernel<<<1, 4 * 32, 0, s>>>(partial, blocks, 4, totals);
  return check_launch("sum_partials_kernel");
}
