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

// ---- decisions in tiles --------------------------------------------------------------------------------
// One CTA takes kDecTile decisions. Every weight row the tile needs — the value MLP's first
// layer (d rows) and every policy head's rows — forms one fused fp32 GEMM
//   out[i, r] = sum_k hidden[i, k] * row_r[k]
// whose weights are staged through shared memory once per CTA in k-slices (instead of once
// per decision), then each decision picks its head's columns. The GEMM computes the logits of
// heads a decision does not use; for the plump heads that is 63 extra rows next to 240.
constexpr int kDecTile = 32;                 // decisions per CTA
constexpr int kDecWarps = 8;                 // warp w owns decisions 4w .. 4w+3 of the tile
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecK = 16;                    // k-slice of staged weights
constexpr int kDecJ = 10;                    // output columns per lane per pass
constexpr int kDecCols = 32 * kDecJ;         // output columns per pass
constexpr int kDecStage = kDecCols * kDecK / kDecThreads;  // staged weights per thread per slice
constexpr int kDecHStride = kDecTile + 4;    // h_s row stride (floats): float4-aligned, fewer conflicts

struct DecideGeometry {
  int n_value;  // rows of the value MLP's first layer in the GEMM (d, or 0 without values)
  int n_rows;   // GEMM output columns: n_value + sum of head widths
  int out_stride;
  int d_pad;    // d rounded up to kDecK
  int head_base[8];
};

__host__ __device__ inline size_t decide_smem_bytes(const DecideGeometry& g, int max_width) {
  return static_cast<size_t>(g.d_pad) * kDecHStride * 4     // h_s
         + static_cast<size_t>(kDecK) * kDecCols * 4        // w_s
         + static_cast<size_t>(kDecTile) * g.out_stride * 4 // out_s
         + static_cast<size_t>(g.n_rows + kDecCols) * 8     // row offsets
         + static_cast<size_t>(kDecWarps) * max_width * 9;  // per-warp logits, probs, mask
}

__global__ void __launch_bounds__(kDecThreads) decide_kernel(cg_heads_desc desc, DecideGeometry g,
                                                              const float* __restrict__ blob,
                                                              const float* __restrict__ hidden,
                                                              const int64_t* __restrict__ hidden_rows,
                                                              int64_t decisions, const int32_t* __restrict__ head_of,
                                                              const uint8_t* __restrict__ legal,
                                                              const double* __restrict__ uniforms, float* logits_out,
                                                              float* probs_out, int64_t* actions_out,
                                                              float* values_out) {
  extern __shared__ __align__(16) unsigned char dec_smem[];
  const int d = desc.d_model, W = desc.max_width;
  float* h_s = reinterpret_cast<float*>(dec_smem);             // [d_pad][kDecHStride], column i = decision
  float* w_s = h_s + static_cast<size_t>(g.d_pad) * kDecHStride;  // [kDecK][kDecCols]
  float* out_s = w_s + kDecK * kDecCols;                         // [kDecTile][out_stride]
  int64_t* row_off = reinterpret_cast<int64_t*>(out_s + static_cast<size_t>(kDecTile) * g.out_stride);
  float* logit_w = reinterpret_cast<float*>(row_off + g.n_rows + kDecCols);  // [kDecWarps][W]
  float* probs_w = logit_w + kDecWarps * W;                                 // [kDecWarps][W]
  uint8_t* mask_w = reinterpret_cast<uint8_t*>(probs_w + kDecWarps * W);  // [kDecWarps][W]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kDecTile;
  const int tile_n = static_cast<int>(decisions - base < kDecTile ? decisions - base : kDecTile);

  // Blob offset of each GEMM row (-1: padding column).
  for (int r = tid; r < g.n_rows + kDecCols; r += kDecThreads) {
    int64_t off = -1;
    if (r < g.n_value) {
      off = desc.value_w1 + static_cast<int64_t>(r) * d;
    } else if (r < g.n_rows) {
      for (int h = 0; h < desc.n_policy; ++h) {
        const int a = r - g.head_base[h];
        if (a >= 0 && a < desc.width[h]) off = desc.weight_offset[h] + static_cast<int64_t>(a) * d;
      }
    }
    row_off[r] = off;
  }
  pdl_wait();  // hidden comes from the kernel before
  pdl_trigger();
  // The tile's hidden rows, transposed (k-major) and zero-padded.
  for (int idx = tid; idx < kDecTile * g.d_pad; idx += kDecThreads) {
    const int i = idx / g.d_pad, k = idx - i * g.d_pad;
    float v = 0.f;
    if (i < tile_n && k < d) {
      const int64_t src = hidden_rows ? hidden_rows[base + i] : base + i;
      v = hidden[src * d + k];
    }
    h_s[k * kDecHStride + i] = v;
  }
  __syncthreads();

  for (int col0 = 0; col0 < g.n_rows; col0 += kDecCols) {
    float acc[4][kDecJ];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int j = 0; j < kDecJ; ++j) acc[r][j] = 0.f;
    float next[kDecStage];
    auto fetch = [&](int k0) {  // element (kk, c) of the slice: c = idx % kDecCols, kk = idx / kDecCols
#pragma unroll
      for (int m = 0; m < kDecStage; ++m) {
        const int idx = tid + m * kDecThreads;
        const int c = idx % kDecCols, kk = idx / kDecCols;
        const int64_t off = row_off[col0 + c];
        next[m] = (off >= 0 && k0 + kk < d) ? __ldg(blob + off + k0 + kk) : 0.f;
      }
    };
    fetch(0);
    for (int k0 = 0; k0 < g.d_pad; k0 += kDecK) {
#pragma unroll
      for (int m = 0; m < kDecStage; ++m) w_s[tid + m * kDecThreads] = next[m];
      __syncthreads();
      if (k0 + kDecK < g.d_pad) fetch(k0 + kDecK);  // in flight during the slice's FMAs
#pragma unroll
      for (int kk = 0; kk < kDecK; ++kk) {
        const float4 hv = *reinterpret_cast<const float4*>(h_s + (k0 + kk) * kDecHStride + 4 * warp);
        const float hr[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int j = 0; j < kDecJ; ++j) {
          const float wv = w_s[kk * kDecCols + lane + 32 * j];
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[r][j] = fmaf(hr[r], wv, acc[r][j]);
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < kDecJ; ++j) {
      const int col = col0 + lane + 32 * j;
      if (col < g.n_rows)
#pragma unroll
        for (int r = 0; r < 4; ++r) out_s[(4 * warp + r) * g.out_stride + col] = acc[r][j];
    }
  }
  __syncthreads();

  // Value MLP: hid = GELU(out[:, :d] + b1) in place, then values = hid W2^T + b2.
  if (g.n_value > 0) {
    const float* b1 = blob + desc.value_b1;
    for (int idx = tid; idx < tile_n * d; idx += kDecThreads) {
      const int i = idx / d, o = idx - i * d;
      float* cell = out_s + i * g.out_stride + o;
      *cell = gelu_erf(*cell + b1[o]);
    }
    __syncthreads();
    const float* W2 = blob + desc.value_w2;
    const float* b2 = blob + desc.value_b2;
    const int V = desc.value_outputs;
    for (int idx = tid; idx < tile_n * V; idx += kDecThreads) {
      const int i = idx / V, o = idx - i * V;
      const float* hid = out_s + i * g.out_stride;
      const float* w2 = W2 + static_cast<int64_t>(o) * d;
      float acc = 0.f;
      for (int k = 0; k < d; ++k) acc = fmaf(hid[k], w2[k], acc);
      values_out[(base + i) * V + o] = acc + b2[o];
    }
  }

  // Policy: warp w takes decisions w, w + 8, ...: its head's columns, mask, sample.
  float* lw = logit_w + warp * W;
  float* pw = probs_w + warp * W;
  uint8_t* mw = mask_w + warp * W;
  for (int i = warp; i < tile_n; i += kDecWarps) {
    const int64_t di = base + i;
    const int head = head_of ? head_of[di] : 0;
    const bool head_ok = head >= 0 && head < desc.n_policy;
    if (!head_ok && lane == 0) raise_fault(0x300);
    const int A = head_ok ? desc.width[head] : 0;
    const float* bh = blob + (head_ok ? desc.bias_offset[head] : 0);
    const float* row = out_s + i * g.out_stride + (head_ok ? g.head_base[head] : 0);
    for (int a = lane; a < W; a += 32) {
      const float logit = a < A ? row[a] + bh[a] : 0.f;
      lw[a] = a < A ? logit : -INFINITY;
      mw[a] = a < A ? legal[di * W + a] : 0;  // entries past the head's width are never legal
      if (logits_out) logits_out[di * W + a] = logit;
    }
    __syncwarp();
    warp_sample(lw, mw, W, uniforms[di], pw, probs_out ? probs_out + di * W : nullptr, actions_out + di);
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
  DecideGeometry g{};
  g.n_value = desc->value_outputs > 0 && values_out ? desc->d_model : 0;
  g.n_rows = g.n_value;
  for (int h = 0; h < desc->n_policy; ++h) {
    g.head_base[h] = g.n_rows;
    g.n_rows += desc->width[h];
  }
  g.out_stride = (g.n_rows + 31) / 32 * 32;
  g.d_pad = (desc->d_model + kDecK - 1) / kDecK * kDecK;
  const size_t smem = decide_smem_bytes(g, desc->max_width);
  CG_REQUIRE(smem <= 227 * 1024, "cg_plump_decide: d_model %d with %d GEMM rows needs %zu bytes of shared memory",
             desc->d_model, g.n_rows, smem);
  static size_t configured[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (configured[device & 63] < smem) {
    cudaError_t err = cudaFuncSetAttribute(decide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "decide_kernel smem: %s", cudaGetErrorString(err));
    configured[device & 63] = smem;
  }
  const unsigned blocks = static_cast<unsigned>((decisions + kDecTile - 1) / kDecTile);
  return launch_pdl("decide_kernel", decide_kernel, dim3(blocks), dim3(kDecThreads), smem,
                    static_cast<cudaStream_t>(stream), *desc, g, heads_blob, hidden, hidden_rows, decisions, head_of,
                    legal, uniforms, logits_out, probs_out, actions_out, values_out);
}
