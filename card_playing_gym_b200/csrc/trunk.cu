// Trunk weight blob, fp32 (CUDA-core) building blocks and the ragged decode orchestration.
//
// Reference: cardgym/nn/trunk.py — Trunk.condition 285-312, _add_ple 318-333,
// forward_ragged 391-429, DecoderBlock._qkv 141-152, forward_ragged 183-223,
// _finish 154-157; cardgym/nn/kv_cache.py write_step 84-105.
#include <cmath>

#include "trunk.h"

namespace cg {

int run_tc_forward(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int64_t batch, int steps,
                   const int64_t* positions, const int64_t* key_lengths, const int64_t* rows, int span, void* k_pool,
                   void* v_pool, int kv_dtype, int64_t capacity, int max_len, bool lookup_blocked,
                   const float* x_in, const float* ple_in, const float* val_in, unsigned char* scratch,
                   int64_t scratch_bytes, const int64_t* readout_offsets, float* hidden_out, int* attn_counters,
                   cudaStream_t s);
int64_t tc_layers_scratch_bytes(const cg_trunk_dims& dims, int64_t batch, int steps);
void tc_input_streams(const cg_trunk_dims& dims, int64_t batch, int steps, unsigned char* scratch, float** x_blk,
                      float** ple_blk, float** val_blk, int64_t* ntiles);
bool tc_layers_available(const cg_trunk_dims& dims);
int tc_pack(const cg_trunk_dims& dims, void* blob, const BlobLayout& L, cudaStream_t stream);
int64_t tc_pack_bytes_ple(const cg_trunk_dims& dims);
int64_t tc_pack_bytes_layer(const cg_trunk_dims& dims);
int tc_condition_ple(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, const float* x,
                     const float* lookup, int64_t lookup_stride, int64_t n, float* ple_out, cudaStream_t stream);

namespace {
constexpr int64_t kAlign = 256;
inline int64_t align_up(int64_t v, int64_t a = kAlign) { return (v + a - 1) / a * a; }
}  // namespace

BlobLayout blob_layout(const cg_trunk_dims& dims) {
  BlobLayout L;
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  const int64_t ple_w = static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim;
  int64_t at = 0;
  auto take = [&](int64_t floats) {
    const int64_t here = at;
    at = align_up(at + floats * 4);
    return here;
  };
  for (int i = 0; i < CG_PART_COUNT; ++i) L.fp32[i] = L.layer_part[i] = -1;
  L.fp32[CG_PART_INPUT_NORM] = dims.input_norm ? take(d) : -1;
  L.fp32[CG_PART_PLE_CONTEXT] = ple_w ? take(ple_w * d) : -1;
  L.fp32[CG_PART_FINAL_W] = take(d);
  L.fp32[CG_PART_FINAL_B] = take(d);
  L.layer_base = at;
  at = 0;
  L.layer_part[CG_PART_LN_ATTN_W] = take(d);
  L.layer_part[CG_PART_LN_ATTN_B] = take(d);
  L.layer_part[CG_PART_QKV] = take(q * d);
  L.layer_part[CG_PART_OUT] = take(d * d);
  L.layer_part[CG_PART_LN_MLP_W] = take(d);
  L.layer_part[CG_PART_LN_MLP_B] = take(d);
  L.layer_part[CG_PART_UP] = take(f * d);
  L.layer_part[CG_PART_UP_B] = take(f);
  L.layer_part[CG_PART_DOWN] = take(d * f);
  L.layer_part[CG_PART_DOWN_B] = take(d);
  L.layer_stride = at;
  at = L.layer_base + L.layer_stride * dims.n_layers;
  L.bf16_ple_context = at;
  at = align_up(at + tc_pack_bytes_ple(dims));
  L.bf16_layer_base = at;
  L.bf16_layer_stride = align_up(tc_pack_bytes_layer(dims));
  at += L.bf16_layer_stride * dims.n_layers;
  // Offsets of the four weight kinds inside a bf16 layer block are fixed by tc_pack.
  L.bf16_qkv = L.bf16_out = L.bf16_up = L.bf16_down = -1;
  L.total = align_up(at);
  return L;
}

// ------------------------------------------------------------------------------------
// fp32 building blocks
// ------------------------------------------------------------------------------------
enum Epilogue { kStore = 0, kGelu = 1, kAccumulate = 2, kCombine = 3 };

// out[r, c] = epilogue(sum_k A[r, k] W[c, k] (+ bias[c])); optional bf16 operand rounding.
// kCombine: out = (addend[r, c] + acc) * scale.
constexpr int kBM = 64, kBN = 64, kBK = 16;

__global__ void __launch_bounds__(256) linear_kernel(const float* __restrict__ A, int64_t lda, const float* __restrict__ W,
                                                    const float* __restrict__ bias, float* out, int64_t ldo,
                                                    const float* __restrict__ addend, int64_t ld_add, float scale,
                                                    int64_t n, int N, int K, int epilogue, int round_operands) {
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Ws[kBK][kBN + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kBM;
  const int col0 = blockIdx.x * kBN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kBK) {
    for (int i = tid; i < kBM * kBK; i += 256) {
      const int r = i / kBK, k = i % kBK;
      const int64_t gr = row0 + r;
      float v = (gr < n && k0 + k < K) ? A[gr * lda + k0 + k] : 0.f;
      As[k][r] = round_operands ? round_bf16(v) : v;
    }
    for (int i = tid; i < kBN * kBK; i += 256) {
      const int c = i / kBK, k = i % kBK;
      const int gc = col0 + c;
      float v = (gc < N && k0 + k < K) ? W[static_cast<int64_t>(gc) * K + k0 + k] : 0.f;
      Ws[k][c] = round_operands ? round_bf16(v) : v;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      float a[4], w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = Ws[k][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty * 4 + i;
    if (r >= n) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = col0 + tx * 4 + j;
      if (c >= N) continue;
      float v = acc[i][j] + (bias ? bias[c] : 0.f);
      float* o = out + r * ldo + c;
      if (epilogue == kGelu) v = gelu_erf(v);
      if (epilogue == kAccumulate) v += *o;
      if (epilogue == kCombine) v = (addend[r * ld_add + c] + acc[i][j]) * scale;
      *o = v;
    }
  }
}

int linear(const float* A, int64_t lda, const float* W, const float* bias, float* out, int64_t ldo, int64_t n, int N,
           int K, int epilogue, bool round_operands, cudaStream_t s, const float* addend = nullptr, int64_t ld_add = 0,
           float scale = 1.f) {
  if (n == 0) return CG_OK;
  dim3 grid((N + kBN - 1) / kBN, static_cast<unsigned>((n + kBM - 1) / kBM));
  linear_kernel<<<grid, 256, 0, s>>>(A, lda, W, bias, out, ldo, addend, ld_add, scale, n, N, K, epilogue,
                                     round_operands ? 1 : 0);
  return check_launch("linear_kernel");
}

// Warp per row: LayerNorm (w, b) or, with b == nullptr and rms != 0, RMSNorm with gain w.
// `index` (optional) gathers input rows: in row = index ? base(r) + index[r] : r.
__global__ void norm_kernel(const float* __restrict__ in, int64_t ld_in, const float* __restrict__ w,
                            const float* __restrict__ b, float* out, int64_t ld_out, int64_t n, int d, float eps,
                            int rms, const int64_t* __restrict__ gather, int gather_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (r >= n) return;
  const int64_t src = gather ? r * gather_stride + gather[r] : r;
  const float* x = in + src * ld_in;
  float sum = 0.f;
  for (int i = lane; i < d; i += 32) sum += rms ? x[i] * x[i] : x[i];
  sum = warp_sum(sum);
  float mean = 0.f, inv;
  if (rms) {
    inv = rsqrtf(sum / d + eps);
  } else {
    mean = sum / d;
    float var = 0.f;
    for (int i = lane; i < d; i += 32) {
      const float c = x[i] - mean;
      var += c * c;
    }
    var = warp_sum(var) / d;
    inv = rsqrtf(var + eps);
  }
  float* y = out + r * ld_out;
  for (int i = lane; i < d; i += 32) y[i] = (x[i] - mean) * inv * w[i] + (b ? b[i] : 0.f);
}

int norm(const float* in, int64_t ld_in, const float* w, const float* b, float* out, int64_t ld_out, int64_t n, int d,
         bool rms, cudaStream_t s, const int64_t* gather = nullptr, int gather_stride = 0) {
  if (n == 0) return CG_OK;
  const int64_t blocks = (n + 7) / 8;
  norm_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(in, ld_in, w, b, out, ld_out, n, d, 1e-5f, rms ? 1 : 0,
                                                            gather, gather_stride);
  return check_launch("norm_kernel");
}

// qkv [B*T, (H + 2 KVH) D] -> q [B, H, T, D] (q_dtype), k/v (+ value embedding) -> pool rows at
// min(positions[b] + t, max_len - 1) (kv_cache.py:84-105 with trunk.py:419-423's clamp).
__global__ void qkv_scatter_kernel(const float* __restrict__ qkv, int64_t batch, int steps, int heads, int kv_heads,
                                   int D, void* q_out, int q_dtype, const float* __restrict__ values, int value_index,
                                   int value_layers, void* k_layer, void* v_layer, int kv_dtype, int max_len,
                                   const int64_t* __restrict__ positions, const int64_t* __restrict__ rows) {
  const int width = (heads + 2 * kv_heads) * D;
  const int64_t total = batch * steps * width;
  const int kvw = kv_heads * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % width);
    const int64_t nt = i / width;
    const int t = static_cast<int>(nt % steps);
    const int64_t b = nt / steps;
    float v = qkv[i];
    if (c < heads * D) {
      const int h = c / D, d = c % D;
      store_from_float(q_out, ((b * heads + h) * steps + t) * D + d, q_dtype, v);
      continue;
    }
    const int cc = c - heads * D;
    const int which = cc / kvw, rem = cc % kvw;
    const int kvh = rem / D, d = rem % D;
    if (which == 1 && value_index >= 0) v += values[(nt * value_layers + value_index) * kvw + rem];
    int64_t pos = positions[b] + t;
    if (pos > max_len - 1) pos = max_len - 1;
    const int64_t row = rows ? rows[b] : b;
    const int64_t dst = ((row * kv_heads + kvh) * max_len + pos) * D + d;
    store_from_float(which ? v_layer : k_layer, dst, kv_dtype, v);
  }
}

// x[nt, j] += ple[nt, layer, j % P] * scale  (trunk.py:318-333, every branch)
__global__ void ple_add_kernel(float* x, const float* __restrict__ ple, int64_t n, int d, int layers, int P, int layer,
                               float scale) {
  const int64_t total = n * d;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / d;
    const int j = static_cast<int>(i % d);
    x[i] += ple[(r * layers + layer) * P + j % P] * scale;
  }
}

// Key lengths (positions + 1) and zeroed per-layer attention work counters.
__global__ void key_lengths_kernel(const int64_t* positions, int64_t* key_lengths, int64_t batch, int* counters,
                                   int n_counters) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < batch) key_lengths[i] = positions[i] + 1;
  if (i < n_counters) counters[i] = 0;
}

inline unsigned grid_for(int64_t total, int threads = 256) {
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  return static_cast<unsigned>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

float ple_scale(int d, int P) {
  if (P == d) return 1.f;
  const int repeats = (d + P - 1) / P;
  return static_cast<float>(1.0 / std::sqrt(static_cast<double>(repeats)));
}

// ------------------------------------------------------------------------------------
// Workspace plan
// ------------------------------------------------------------------------------------
struct StepWorkspace {
  float* x;       // [NT, d] residual stream
  float* h;       // [NT, max(q, f, d)]
  float* h2;      // [NT, f]
  void* q;        // [B, H, T, D] fp32 or cache dtype
  float* attn;    // [B, T, H, D]
  int64_t* key_lengths;  // [B]
  int* attn_counters;    // [kMaxLayers]: one work counter per layer's attention launch
  unsigned char* tc;     // tensor-core path scratch
  int64_t tc_bytes;
  int64_t total;
};

StepWorkspace plan_step(const cg_trunk_dims& dims, int64_t batch, int steps, int precision, unsigned char* base) {
  StepWorkspace w{};
  const int64_t nt = batch * steps;
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  int64_t at = 0;
  auto take = [&](int64_t bytes) {
    unsigned char* here = base ? base + at : nullptr;
    at = align_up(at + bytes);
    return here;
  };
  w.x = reinterpret_cast<float*>(take(nt * d * 4));
  w.key_lengths = reinterpret_cast<int64_t*>(take(batch * 8));
  w.attn_counters = reinterpret_cast<int*>(take(64 * sizeof(int)));
  if (precision == CG_PREC_BF16 && tc_layers_available(dims)) {
    w.tc_bytes = tc_layers_scratch_bytes(dims, batch, steps);
    w.tc = take(w.tc_bytes);
  } else {
    const int64_t hw = q > f ? (q > d ? q : d) : (f > d ? f : d);
    w.h = reinterpret_cast<float*>(take(nt * hw * 4));
    w.h2 = reinterpret_cast<float*>(take(nt * f * 4));
    w.q = take(nt * d * 4);
    w.attn = reinterpret_cast<float*>(take(nt * d * 4));
  }
  w.total = at;
  return w;
}

// The tensor-core scratch inside a step workspace (null when the step takes the CUDA-core path).
unsigned char* step_tc_scratch(const cg_trunk_dims& dims, int64_t batch, int steps, int precision, void* workspace) {
  return plan_step(dims, batch, steps, precision, static_cast<unsigned char*>(workspace)).tc;
}

int check_dims(const cg_trunk_dims* dims) {
  CG_REQUIRE(dims, "NULL trunk dims");
  CG_REQUIRE(dims->d_model > 0 && dims->n_layers > 0 && dims->n_heads > 0 && dims->n_kv_heads > 0 && dims->d_ff > 0,
             "trunk dims must be positive");
  CG_REQUIRE(dims->d_model % dims->n_heads == 0, "d_model %d must divide by n_heads %d", dims->d_model, dims->n_heads);
  CG_REQUIRE(dims->n_heads % dims->n_kv_heads == 0, "n_kv_heads must divide n_heads");
  CG_REQUIRE(dims->n_layers <= 64, "at most 64 layers");
  CG_REQUIRE(dims->per_layer_dim >= 0, "per_layer_dim must be non-negative");
  return CG_OK;
}

// The layer loop over a residual stream x already in the workspace (fp32 path).
int run_fp32_layers(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int64_t batch, int steps,
                    const int64_t* positions, const int64_t* rows, int span, void* k_pool, void* v_pool, int kv_dtype,
                    int64_t capacity, int max_len, const float* ple, const float* values, StepWorkspace& w,
                    bool bf16, cudaStream_t s) {
  const int d = dims.d_model, f = dims.d_ff, H = dims.n_heads, KVH = dims.n_kv_heads, D = head_dim(dims);
  const int qw = qkv_width(dims);
  const int64_t nt = batch * steps;
  const int64_t layer_elems = capacity * KVH * static_cast<int64_t>(max_len) * D;
  const int esize = dtype_size(kv_dtype);
  const int q_dtype = kv_dtype;  // q is cast to the cache dtype (trunk.py:222)
  const int nvl = value_layer_count(dims);
  int rc;
  for (int layer = 0; layer < dims.n_layers; ++layer) {
    void* k_layer = static_cast<unsigned char*>(k_pool) + layer * layer_elems * esize;
    void* v_layer = static_cast<unsigned char*>(v_pool) + layer * layer_elems * esize;
    if ((rc = norm(w.x, d, part(blob, L, CG_PART_LN_ATTN_W, layer), part(blob, L, CG_PART_LN_ATTN_B, layer), w.h, d, nt,
                   d, false, s)))
      return rc;
    if ((rc = linear(w.h, d, part(blob, L, CG_PART_QKV, layer), nullptr, w.h2, qw, nt, qw, d, kStore, bf16, s)))
      return rc;
    qkv_scatter_kernel<<<grid_for(nt * qw), 256, 0, s>>>(w.h2, batch, steps, H, KVH, D, w.q, q_dtype, values,
                                                          value_index(dims, layer), nvl, k_layer, v_layer, kv_dtype,
                                                          max_len, positions, rows);
    if ((rc = check_launch("qkv_scatter_kernel"))) return rc;
    AttnParams p{};
    p.q = w.q;
    p.q_dtype = q_dtype;
    p.q_st = D;
    p.q_sh = static_cast<int64_t>(steps) * D;
    p.q_sb = static_cast<int64_t>(H) * steps * D;
    p.k = k_layer;
    p.v = v_layer;
    p.kv_dtype = kv_dtype;
    p.kv_pos = D;
    p.kv_head = static_cast<int64_t>(max_len) * D;
    p.kv_row = static_cast<int64_t>(KVH) * max_len * D;
    p.rows = rows;
    p.lengths = w.key_lengths;
    p.counter = w.attn_counters + layer;
    p.batch = batch;
    p.heads = H;
    p.kv_heads = KVH;
    p.steps = steps;
    p.group = H / KVH;
    p.head_dim = D;
    p.span = span;
    p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
    p.out = w.attn;
    p.out_dtype = CG_F32;
    // attention output as [B, T, H, D]: row-token major for the out projection
    p.o_st = static_cast<int64_t>(H) * D;
    p.o_sh = D;
    p.o_sb = static_cast<int64_t>(steps) * H * D;
    if ((rc = run_attention(p, s))) return rc;
    if ((rc = linear(w.attn, d, part(blob, L, CG_PART_OUT, layer), nullptr, w.x, d, nt, d, d, kAccumulate, bf16, s)))
      return rc;
    if ((rc = norm(w.x, d, part(blob, L, CG_PART_LN_MLP_W, layer), part(blob, L, CG_PART_LN_MLP_B, layer), w.h, d, nt,
                   d, false, s)))
      return rc;
    if ((rc = linear(w.h, d, part(blob, L, CG_PART_UP, layer), part(blob, L, CG_PART_UP_B, layer), w.h2, f, nt, f, d,
                     kGelu, bf16, s)))
      return rc;
    if ((rc = linear(w.h2, f, part(blob, L, CG_PART_DOWN, layer), part(blob, L, CG_PART_DOWN_B, layer), w.x, d, nt, d,
                     f, kAccumulate, bf16, s)))
      return rc;
    if (dims.per_layer_dim) {
      ple_add_kernel<<<grid_for(nt * d), 256, 0, s>>>(w.x, ple, nt, d, dims.n_layers, dims.per_layer_dim, layer,
                                                      ple_scale(d, dims.per_layer_dim));
      if ((rc = check_launch("ple_add_kernel"))) return rc;
    }
  }
  return CG_OK;
}

// The layer loop from either conditioned inputs (x_in, ple, values) or, on the tensor-core
// path, the raw field lookup already written into the step's scratch in blocked layout by the
// lookup kernel (lookup_blocked: conditioning runs inside the first kernel).
// x_in_workspace: x_in already is the step workspace's residual buffer (fp32 path only).
int forward_ragged_impl(const cg_trunk_dims* dims_p, const void* blob, const float* x_in, const float* ple,
                        const float* values, int64_t batch, int steps, const int64_t* positions,
                        const int64_t* readout_offsets, const int64_t* rows, int span, void* k_pool, void* v_pool,
                        int kv_dtype, int64_t capacity, int max_len, int precision, void* workspace,
                        int64_t workspace_bytes, float* hidden_out, cudaStream_t s, bool x_in_workspace,
                        bool lookup_blocked) {
  int rc;
  if ((rc = check_dims(dims_p))) return rc;
  const cg_trunk_dims& dims = *dims_p;
  CG_REQUIRE(precision == CG_PREC_FP32 || precision == CG_PREC_BF16, "unknown precision %d", precision);
  CG_REQUIRE(valid_dtype(kv_dtype), "bad kv dtype");
  CG_REQUIRE(batch >= 0 && steps > 0, "bad batch/steps");
  CG_REQUIRE(max_len > 0 && capacity > 0, "bad pool shape");
  if (batch == 0) return CG_OK;
  CG_REQUIRE(blob && positions && readout_offsets && k_pool && v_pool && hidden_out && workspace, "NULL pointer");
  CG_REQUIRE(lookup_blocked || !dims.per_layer_dim || ple, "this trunk expects a per-layer embedding lookup");
  CG_REQUIRE(lookup_blocked || !dims.value_layers || values, "this trunk expects a value-embedding lookup");
  if (span > max_len) span = max_len;
  StepWorkspace w = plan_step(dims, batch, steps, precision, static_cast<unsigned char*>(workspace));
  if (workspace_bytes < w.total)
    return set_error(CG_ERR_WORKSPACE, "trunk step workspace %lld < %lld bytes", (long long)workspace_bytes,
                     (long long)w.total);
  const BlobLayout L = blob_layout(dims);
  const int64_t nt = batch * steps;
  key_lengths_kernel<<<static_cast<unsigned>((batch + 255) / 256), 256, 0, s>>>(positions, w.key_lengths, batch,
                                                                                  w.attn_counters, 64);
  if ((rc = check_launch("key_lengths_kernel"))) return rc;
  if (precision == CG_PREC_BF16 && tc_layers_available(dims)) {
    return run_tc_forward(dims, blob, L, batch, steps, positions, w.key_lengths, rows, span, k_pool, v_pool, kv_dtype,
                          capacity, max_len, lookup_blocked, x_in, ple, values, w.tc, w.tc_bytes,
                          readout_offsets, hidden_out, w.attn_counters, s);
  }
  CG_REQUIRE(!lookup_blocked, "internal: the CUDA-core path takes conditioned inputs");
  if (!x_in_workspace) {
    cudaError_t err = cudaMemcpyAsync(w.x, x_in, nt * dims.d_model * sizeof(float), cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "copy x: %s", cudaGetErrorString(err));
  }
  rc = run_fp32_layers(dims, blob, L, batch, steps, positions, rows, span, k_pool, v_pool, kv_dtype, capacity,
                       max_len, ple, values, w, precision == CG_PREC_BF16, s);
  if (rc) return rc;
  // final LayerNorm at each row's readout token only (trunk.py:429)
  return norm(w.x, dims.d_model, part(blob, L, CG_PART_FINAL_W, 0), part(blob, L, CG_PART_FINAL_B, 0), hidden_out,
              dims.d_model, batch, dims.d_model, false, s, readout_offsets, steps);
}

__global__ void f32_to_bf16_kernel(const float* in, __nv_bfloat16* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

}  // namespace cg

// ------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------
extern "C" int64_t cg_trunk_blob_bytes(const cg_trunk_dims* dims) {
  if (cg::check_dims(dims)) return -1;
  return cg::blob_layout(*dims).total;
}

extern "C" int64_t cg_trunk_part_offset(const cg_trunk_dims* dims, int which, int layer) {
  if (cg::check_dims(dims) || which < 0 || which >= CG_PART_COUNT) return -1;
  const cg::BlobLayout L = cg::blob_layout(*dims);
  if (which <= CG_PART_FINAL_B) return L.fp32[which];
  if (layer < 0 || layer >= dims->n_layers) return -1;
  return L.layer_base + layer * L.layer_stride + L.layer_part[which];
}

extern "C" int cg_trunk_prepare(const cg_trunk_dims* dims, void* blob, void* stream) {
  int rc;
  if ((rc = cg::check_dims(dims))) return rc;
  CG_REQUIRE(blob, "cg_trunk_prepare: NULL blob");
  return cg::tc_pack(*dims, blob, cg::blob_layout(*dims), static_cast<cudaStream_t>(stream));
}

extern "C" int64_t cg_trunk_step_workspace_bytes(const cg_trunk_dims* dims, int64_t batch, int steps, int precision) {
  if (cg::check_dims(dims)) return -1;
  return cg::plan_step(*dims, batch, steps, precision, nullptr).total;
}

extern "C" int cg_trunk_forward_ragged(const cg_trunk_dims* dims, const void* blob, const float* x, const float* ple,
                                       const float* values, int64_t batch, int steps, const int64_t* positions,
                                       const int64_t* readout_offsets, const int64_t* rows, int span, void* k_pool,
                                       void* v_pool, int kv_dtype, int64_t capacity, int max_len, int precision,
                                       void* workspace, int64_t workspace_bytes, float* hidden_out, void* stream) {
  if (batch > 0 && !x) return cg::set_error(CG_ERR_ARGUMENT, "cg_trunk_forward_ragged: NULL x");
  return cg::forward_ragged_impl(dims, blob, x, ple, values, batch, steps, positions, readout_offsets, rows, span,
                                 k_pool, v_pool, kv_dtype, capacity, max_len, precision, workspace, workspace_bytes,
                                 hidden_out, static_cast<cudaStream_t>(stream), false, false);
}

extern "C" int cg_trunk_condition(const cg_trunk_dims* dims_p, const void* blob, const float* lookup, int64_t n,
                                  float* x_out, float* ple_out, float* values_out, int precision, void* stream) {
  using namespace cg;
  int rc;
  if ((rc = check_dims(dims_p))) return rc;
  const cg_trunk_dims& dims = *dims_p;
  if (n == 0) return CG_OK;
  CG_REQUIRE(blob && lookup && x_out, "cg_trunk_condition: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const BlobLayout L = blob_layout(dims);
  const int d = dims.d_model;
  const int ple_w = dims.n_layers * dims.per_layer_dim;
  const int val_w = value_layer_count(dims) * dims.n_kv_heads * head_dim(dims);
  const int64_t width = d + ple_w + val_w;
  // x = RMSNorm(lookup[:, :d]) (trunk.py:297-298)
  if (dims.input_norm) {
    if ((rc = norm(lookup, width, part(blob, L, CG_PART_INPUT_NORM, 0), nullptr, x_out, d, n, d, true, s))) return rc;
  } else {
    cudaError_t err = cudaMemcpy2DAsync(x_out, d * 4, lookup, width * 4, d * 4, n, cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "copy x: %s", cudaGetErrorString(err));
  }
  if (ple_w) {
    CG_REQUIRE(ple_out, "cg_trunk_condition: NULL ple_out");
    // ple = (lookup_ple + W_c x) / sqrt(2) (trunk.py:301-306)
    if (precision == CG_PREC_BF16 && tc_layers_available(dims)) {
      rc = tc_condition_ple(dims, blob, L, x_out, lookup + d, width, n, ple_out, s);
    } else {
      rc = linear(x_out, d, part(blob, L, CG_PART_PLE_CONTEXT, 0), nullptr, ple_out, ple_w, n, ple_w, d, kCombine,
                  precision == CG_PREC_BF16, s, lookup + d, width, static_cast<float>(1.0 / std::sqrt(2.0)));
    }
    if (rc) return rc;
  }
  if (val_w) {
    CG_REQUIRE(values_out, "cg_trunk_condition: NULL values_out");
    cudaError_t err = cudaMemcpy2DAsync(values_out, val_w * 4, lookup + d + ple_w, width * 4, val_w * 4, n,
                                        cudaMemcpyDeviceToDevice, s);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "copy values: %s", cudaGetErrorString(err));
  }
  return CG_OK;
}
