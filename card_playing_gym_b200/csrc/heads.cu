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
// The exp is numpy's float32 exp and the sum numpy's pairwise order over the numpy row
// (numpy_math.cuh), the division and the running cumsum are single float32 roundings and
// the comparison is in float64, so for the same logits and uniforms the probabilities and
// the draws are bit-identical to the reference's numpy sampler.
#include "common.cuh"
#include "numpy_math.cuh"

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
  for (int j = lane; j < width; j += 32) probs_s[j] = mask[j] ? numpy_expf(__fsub_rn(logits[j], peak)) : 0.f;
  __syncwarp();
  const float total = numpy_row_sum(probs_s, width);  // the numpy row is the whole width
  __syncwarp();
  for (int j = lane; j < width; j += 32) {
    const float p = __fdiv_rn(probs_s[j], total);
    probs_s[j] = p;
    if (probs_out) probs_out[j] = p;
  }
  __syncwarp();
  if (lane == 0) {
    float cdf = 0.f;
    int below = 0;
    for (int j = 0; j < width; ++j) {
      cdf = __fadd_rn(cdf, probs_s[j]);
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
// layer and every policy head — forms the columns of one fp32 GEMM
//   out[i, r] = sum_k hidden[i, k] * row_r[k]
// whose weights stream through shared memory in k-slices (a three-stage cp.async ring of
// 16-byte row segments, started before the kernel before has finished: the weights do not
// depend on it), once per CTA instead of once per decision; each decision then picks its
// head's columns. The GEMM computes the logits of heads a decision does not use; for the
// plump heads that is 63 extra rows next to 240. Each thread owns 8 decisions x 5 columns,
// so one 16-byte weight read feeds 32 FMAs and every output sums over k in order.
constexpr int kDecTile = 32;                              // decisions per CTA
constexpr int kDecWarps = 8;
constexpr int kDecThreads = kDecWarps * 32;
constexpr int kDecGroups = 4;                             // warp w: decision group w % 4 ...
constexpr int kDecGroupRows = kDecTile / kDecGroups;      // ... of 8 decisions,
constexpr int kDecHalves = kDecWarps / kDecGroups;        // column half w / 4 ...
constexpr int kDecJ = 5;                                  // ... of 5 columns per lane
constexpr int kDecCols = 32 * kDecJ * kDecHalves;         // GEMM columns per pass
constexpr int kDecK = 16;                                 // k-slice per stage
constexpr int kDecKStride = kDecK + 4;                    // w_s row (floats): 80-byte rows keep 16-byte reads conflict-free
constexpr int kDecStages = 3;
constexpr int kDecHStride = kDecTile + 4;                 // h_s row stride (floats), 16-byte aligned rows
constexpr int kDecStageFloats = kDecCols * kDecKStride;
constexpr int kDecSegments = kDecCols * (kDecK / 4);      // 16-byte segments per slice

static_assert(kDecGroupRows == 8, "the GEMM reads a group's hidden values as two float4");
static_assert(kDecK % 4 == 0 && kDecSegments % kDecThreads == 0, "whole segments per thread");
static_assert(kDecTile <= 32 * kDecWarps, "one CDF thread per decision");

struct DecideGeometry {
  int n_value;  // rows of the value MLP's first layer in the GEMM (d, or 0 without values)
  int n_rows;   // GEMM output columns: n_value + sum of head widths
  int out_stride;
  int d_pad;    // d rounded up to kDecK
  int n_w2;     // floats of the value MLP's second layer staged in shared memory (0 without values)
  int head_base[8];
};

__host__ __device__ inline size_t decide_smem_bytes(const DecideGeometry& g, int max_width) {
  return static_cast<size_t>(g.d_pad) * kDecHStride * 4         // h_s
         + static_cast<size_t>(kDecStages) * kDecStageFloats * 4  // w_s ring
         + static_cast<size_t>(kDecTile) * g.out_stride * 4     // out_s
         + static_cast<size_t>(g.n_rows + kDecCols) * 12        // row offsets and column biases
         + static_cast<size_t>(kDecTile) * 8                    // uniforms
         + static_cast<size_t>(g.n_w2) * 4                      // value second layer
         + static_cast<size_t>(kDecTile) * max_width * 5        // per-decision probabilities and mask
         + static_cast<size_t>(kDecTile) * 8;                   // per-decision head and last legal index
}

__device__ __forceinline__ void dec_cp_async16(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void dec_cp_async4(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}

// kVec: the blob and hidden are 16-byte aligned, d % 4 == 0 and every weight row offset is a
// multiple of 4 floats, so weights and hidden rows move in 16-byte pieces.
template <bool kVec>
__global__ void __launch_bounds__(kDecThreads, 1) decide_kernel(cg_heads_desc desc, DecideGeometry g,
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
  float* h_s = reinterpret_cast<float*>(dec_smem);                 // [d_pad][kDecHStride], column i = decision
  float* w_s = h_s + static_cast<size_t>(g.d_pad) * kDecHStride;   // [kDecStages][kDecCols][kDecKStride]
  float* out_s = w_s + kDecStages * kDecStageFloats;               // [kDecTile][out_stride]
  int64_t* row_off = reinterpret_cast<int64_t*>(out_s + static_cast<size_t>(kDecTile) * g.out_stride);
  double* u_s = reinterpret_cast<double*>(row_off + g.n_rows + kDecCols);  // [kDecTile]
  float* col_bias = reinterpret_cast<float*>(u_s + kDecTile);             // [n_rows + kDecCols]
  float* w2_s = col_bias + g.n_rows + kDecCols;                           // [value_outputs][d]
  float* p_s = w2_s + g.n_w2;                                             // [kDecTile][W]
  int* last_s = reinterpret_cast<int*>(p_s + kDecTile * W);               // [kDecTile]
  int* head_s = last_s + kDecTile;                                        // [kDecTile]
  uint8_t* m_s = reinterpret_cast<uint8_t*>(head_s + kDecTile);           // [kDecTile][W], legal bytes
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kDecTile;
  const int tile_n = static_cast<int>(decisions - base < kDecTile ? decisions - base : kDecTile);
  const int n_slices = g.d_pad / kDecK;

  // Blob offset (-1: padding column) and bias of each GEMM row; the value MLP's second layer.
  for (int r = tid; r < g.n_rows + kDecCols; r += kDecThreads) {
    int64_t off = -1;
    float bias = 0.f;
    if (r < g.n_value) {
      off = desc.value_w1 + static_cast<int64_t>(r) * d;
      bias = blob[desc.value_b1 + r];
    } else if (r < g.n_rows) {
      for (int h = 0; h < desc.n_policy; ++h) {
        const int a = r - g.head_base[h];
        if (a >= 0 && a < desc.width[h]) {
          off = desc.weight_offset[h] + static_cast<int64_t>(a) * d;
          bias = blob[desc.bias_offset[h] + a];
        }
      }
    }
    row_off[r] = off;
    col_bias[r] = bias;
  }
  for (int idx = tid; idx < g.n_w2; idx += kDecThreads) w2_s[idx] = blob[desc.value_w2 + idx];
  __syncthreads();

  // Slice `slice` of pass `col0` into ring stage `stage`: segment q holds k-values
  // [k0 + 4 (q % 4), +4) of column q / 4 (four threads read a row's 64 contiguous bytes).
  auto issue = [&](int col0, int slice, int stage) {
    float* dst = w_s + stage * kDecStageFloats;
    const int k0 = slice * kDecK;
#pragma unroll
    for (int m = 0; m < kDecSegments / kDecThreads; ++m) {
      const int q = tid + m * kDecThreads, c = q >> 2, part = q & 3;
      const int64_t off = row_off[col0 + c];
      const int k = k0 + 4 * part;
      float* d4 = dst + c * kDecKStride + 4 * part;
      if (kVec) {
        const bool valid = off >= 0 && k < d;
        dec_cp_async16(d4, valid ? blob + off + k : blob, valid);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool valid = off >= 0 && k + e < d;
          dec_cp_async4(d4 + e, valid ? blob + off + k + e : blob, valid);
        }
      }
    }
  };
  auto prologue = [&](int col0) {
#pragma unroll
    for (int st = 0; st < kDecStages - 1; ++st) {
      if (st < n_slices) issue(col0, st, st);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  };
  prologue(0);  // the weights do not depend on the kernel before
  pdl_wait();   // hidden comes from the kernel before
  pdl_trigger();

  // The tile's heads, uniforms and legal bytes (rows of W, contiguous across the tile).
  for (int i = tid; i < tile_n; i += kDecThreads) {
    head_s[i] = head_of ? head_of[base + i] : 0;
    u_s[i] = uniforms[base + i];
  }
  for (int idx = tid; idx < tile_n * W; idx += kDecThreads) m_s[idx] = legal[base * W + idx];

  // The tile's hidden rows, transposed (k-major) and zero-padded.
  if (kVec) {
    const int d4 = d / 4, p4 = g.d_pad / 4;
    for (int idx = tid; idx < kDecTile * p4; idx += kDecThreads) {
      const int i = idx / p4, k4 = idx - i * p4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < tile_n && k4 < d4) {
        const int64_t src = hidden_rows ? hidden_rows[base + i] : base + i;
        v = reinterpret_cast<const float4*>(hidden + src * d)[k4];
      }
      float* col = h_s + 4 * k4 * kDecHStride + i;
      col[0] = v.x;
      col[kDecHStride] = v.y;
      col[2 * kDecHStride] = v.z;
      col[3 * kDecHStride] = v.w;
    }
  } else {
    for (int idx = tid; idx < kDecTile * g.d_pad; idx += kDecThreads) {
      const int i = idx / g.d_pad, k = idx - i * g.d_pad;
      float v = 0.f;
      if (i < tile_n && k < d) {
        const int64_t src = hidden_rows ? hidden_rows[base + i] : base + i;
        v = hidden[src * d + k];
      }
      h_s[k * kDecHStride + i] = v;
    }
  }

  const int grp = warp % kDecGroups, half = warp / kDecGroups;
  for (int col0 = 0; col0 < g.n_rows; col0 += kDecCols) {
    if (col0 > 0) {
      __syncthreads();  // every warp is done with the ring before the next pass refills it
      prologue(col0);
    }
    float acc[kDecGroupRows][kDecJ];
#pragma unroll
    for (int r = 0; r < kDecGroupRows; ++r)
#pragma unroll
      for (int j = 0; j < kDecJ; ++j) acc[r][j] = 0.f;
    for (int sl = 0; sl < n_slices; ++sl) {
      asm volatile("cp.async.wait_group %0;" ::"n"(kDecStages - 2) : "memory");
      __syncthreads();  // slice sl (and, on the first pass, h_s) is in place; stage sl - 1 is free
      if (sl + kDecStages - 1 < n_slices) issue(col0, sl + kDecStages - 1, (sl + kDecStages - 1) % kDecStages);
      asm volatile("cp.async.commit_group;" ::: "memory");
      const float* ws = w_s + (sl % kDecStages) * kDecStageFloats + (half * 32 * kDecJ + lane) * kDecKStride;
      const float* hs = h_s + sl * kDecK * kDecHStride + kDecGroupRows * grp;
#pragma unroll
      for (int kq = 0; kq < kDecK / 4; ++kq) {
        float4 w[kDecJ];
#pragma unroll
        for (int j = 0; j < kDecJ; ++j) w[j] = *reinterpret_cast<const float4*>(ws + j * 32 * kDecKStride + 4 * kq);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float* hk = hs + (4 * kq + kk) * kDecHStride;
          const float4 h0 = *reinterpret_cast<const float4*>(hk);
          const float4 h1 = *reinterpret_cast<const float4*>(hk + 4);
          const float hv[kDecGroupRows] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
          for (int j = 0; j < kDecJ; ++j) {
            const float wv = kk == 0 ? w[j].x : kk == 1 ? w[j].y : kk == 2 ? w[j].z : w[j].w;
#pragma unroll
            for (int r = 0; r < kDecGroupRows; ++r) acc[r][j] = fmaf(hv[r], wv, acc[r][j]);
          }
        }
      }
    }
    // Value columns leave as GELU(. + b1) (the value MLP's hidden layer); policy columns as
    // logits (. + the head's bias).
#pragma unroll
    for (int j = 0; j < kDecJ; ++j) {
      const int col = col0 + half * 32 * kDecJ + lane + 32 * j;
      if (col < g.n_rows) {
        const bool value = col < g.n_value;
        const float bias = col_bias[col];
#pragma unroll
        for (int r = 0; r < kDecGroupRows; ++r) {
          const float a = acc[r][j] + bias;
          out_s[(kDecGroupRows * grp + r) * g.out_stride + col] = value ? gelu_erf(a) : a;
        }
      }
    }
  }
  __syncthreads();

  // Values: one warp per decision, up to eight outputs at a time, lanes split k.
  if (g.n_value > 0) {
    const float* b2 = blob + desc.value_b2;
    const int V = desc.value_outputs;
    for (int i = warp; i < tile_n; i += kDecWarps) {
      const float* hid = out_s + i * g.out_stride;
      for (int o0 = 0; o0 < V; o0 += 8) {
        float acc[8];
#pragma unroll
        for (int o = 0; o < 8; ++o) acc[o] = 0.f;
        for (int k = lane; k < d; k += 32) {
          const float h = hid[k];
#pragma unroll
          for (int o = 0; o < 8; ++o)
            if (o0 + o < V) acc[o] = fmaf(h, w2_s[(o0 + o) * d + k], acc[o]);
        }
#pragma unroll
        for (int o = 0; o < 8; ++o) acc[o] = warp_sum(acc[o]);
        if (lane < 8 && o0 + lane < V) {
          float v = acc[0];
#pragma unroll
          for (int o = 1; o < 8; ++o) v = lane == o ? acc[o] : v;
          values_out[(base + i) * V + o0 + lane] = v + b2[o0 + lane];
        }
      }
    }
  }

  // Policy: warp w takes decisions w, w + kDecWarps, ...: its head's columns and mask, the
  // legal max, exp and normalisation (the same per-lane order as warp_sample).
  for (int i = warp; i < tile_n; i += kDecWarps) {
    const int64_t di = base + i;
    const int head = head_s[i];
    const bool head_ok = head >= 0 && head < desc.n_policy;
    if (!head_ok && lane == 0) raise_fault(0x300);
    const int A = head_ok ? desc.width[head] : 0;
    const float* row = out_s + i * g.out_stride + (head_ok ? g.head_base[head] : 0);
    float* lp = p_s + i * W;
    uint8_t* lm = m_s + i * W;
    float peak = -INFINITY;
    int last_legal = -1;
    for (int a = lane; a < W; a += 32) {
      const float logit = a < A ? row[a] : 0.f;
      const uint8_t m = a < A ? lm[a] : 0;  // entries past the head's width are never legal
      if (logits_out) logits_out[di * W + a] = logit;
      lp[a] = a < A ? logit : -INFINITY;
      lm[a] = m;
      if (m) {
        peak = fmaxf(peak, logit);
        last_legal = a;
      }
    }
    peak = warp_max(peak);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) last_legal = max(last_legal, __shfl_xor_sync(0xffffffffu, last_legal, o));
    for (int a = lane; a < W; a += 32) lp[a] = lm[a] ? numpy_expf(__fsub_rn(lp[a], peak)) : 0.f;
    __syncwarp();
    // The reference samples a head's decisions as rows of the head's own width
    // (selfplay.py:532-545: plump's legal vectors span the whole head), so the sum runs
    // over A entries in numpy's order; the entries past A are zero.
    const float total = numpy_row_sum(lp, A);
    __syncwarp();
    for (int a = lane; a < W; a += 32) {
      const float p = __fdiv_rn(lp[a], total);
      lp[a] = p;
      if (probs_out) probs_out[di * W + a] = p;
    }
    if (lane == 0) last_s[i] = last_legal;
  }
  __syncthreads();

  // Draws: one thread per decision walks its CDF in order (float32 running sum, compared in
  // float64 with the uniform). The running sum never decreases, so the count of steps below
  // u ends at the first step at or above it.
  if (lane < kDecTile / kDecWarps) {
    const int i = warp + kDecWarps * lane;
    if (i < tile_n) {
      const int64_t di = base + i;
      const double u = u_s[i];
      const float* lp = p_s + i * W;
      float cdf = 0.f;
      int below = 0;
      bool done = false;
      for (; below + 4 <= W && !done; below += 4) {  // four probabilities read ahead of the sums
        const float p0 = lp[below], p1 = lp[below + 1], p2 = lp[below + 2], p3 = lp[below + 3];
        cdf = __fadd_rn(cdf, p0);
        if (!(static_cast<double>(cdf) < u)) { done = true; break; }
        cdf = __fadd_rn(cdf, p1);
        if (!(static_cast<double>(cdf) < u)) { below += 1; done = true; break; }
        cdf = __fadd_rn(cdf, p2);
        if (!(static_cast<double>(cdf) < u)) { below += 2; done = true; break; }
        cdf = __fadd_rn(cdf, p3);
        if (!(static_cast<double>(cdf) < u)) { below += 3; done = true; break; }
      }
      for (; below < W && !done; ++below) {
        cdf = __fadd_rn(cdf, lp[below]);
        if (!(static_cast<double>(cdf) < u)) break;
      }
      const int last_legal = last_s[i];
      int drawn = last_legal < 0 ? 0 : min(below, last_legal);
      if (last_legal >= 0 && !m_s[i * W + drawn]) drawn = last_legal;
      actions_out[di] = drawn;
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
  DecideGeometry g{};
  g.n_value = desc->value_outputs > 0 && values_out ? desc->d_model : 0;
  g.n_rows = g.n_value;
  for (int h = 0; h < desc->n_policy; ++h) {
    g.head_base[h] = g.n_rows;
    g.n_rows += desc->width[h];
  }
  g.out_stride = (g.n_rows + 31) / 32 * 32;
  g.d_pad = (desc->d_model + kDecK - 1) / kDecK * kDecK;
  g.n_w2 = g.n_value > 0 ? desc->value_outputs * desc->d_model : 0;
  const size_t smem = decide_smem_bytes(g, desc->max_width);
  CG_REQUIRE(smem <= 227 * 1024, "cg_plump_decide: d_model %d with %d GEMM rows needs %zu bytes of shared memory",
             desc->d_model, g.n_rows, smem);
  bool vec = reinterpret_cast<uintptr_t>(heads_blob) % 16 == 0 && reinterpret_cast<uintptr_t>(hidden) % 16 == 0 &&
             desc->d_model % 4 == 0 && (g.n_value == 0 || desc->value_w1 % 4 == 0);
  for (int h = 0; h < desc->n_policy; ++h) vec = vec && desc->weight_offset[h] % 4 == 0;
  static size_t configured[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (configured[device & 63] < smem) {
    for (auto kernel : {decide_kernel<true>, decide_kernel<false>}) {
      cudaError_t err =
          cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "decide_kernel smem: %s", cudaGetErrorString(err));
    }
    configured[device & 63] = smem;
  }
  const unsigned blocks = static_cast<unsigned>((decisions + kDecTile - 1) / kDecTile);
  const auto launch = [&](auto kernel) {
    return launch_pdl("decide_kernel", kernel, dim3(blocks), dim3(kDecThreads), smem,
                      static_cast<cudaStream_t>(stream), *desc, g, heads_blob, hidden, hidden_rows, decisions,
                      head_of, legal, uniforms, logits_out, probs_out, actions_out, values_out);
  };
  return vec ? launch(decide_kernel<true>) : launch(decide_kernel<false>);
}
