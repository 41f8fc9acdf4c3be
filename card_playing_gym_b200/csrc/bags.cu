// One-hot field bags: the piquet (and any fixed-field) token lookup.
//
// Reference: cardgym/games/piquet/model.py:255-264 (`_onehot_bags`) and 323-345
// (`PiquetEmbedding.forward`): ids = tokens[..., :NUM_FIELDS] + offsets, then every table's
// field sums as ONE GEMM of the tokens' one-hot rows against the tables side by side,
//   hot = zeros(N, rows).scatter_(1, ids, 1.0);  sums = hot @ cat(tables, 1).to(dtype)
// in the autocast dtype (fp16/bf16, fp32 accumulation, each sum rounded once) or fp32.
//
// Here the one-hot product is a gather-sum: each DISTINCT row a token selects is added once
// (scatter_ writes 1.0, so an id repeated within a token counts once), in field order, in
// fp32, from the table in its own dtype, and the sum is rounded once to that dtype. An id
// outside [0, rows) sets the device fault word to 0x210 (the reference's scatter_ raises an
// index error) and selects nothing.
//
// One warp per token: lanes resolve the token's field ids (one field per lane), drop
// repeats with __match_any_sync, then stride the row in 16-byte units; the table (a few MB)
// stays L2-resident, every unit is a coalesced 512-byte warp read per selected row.
#include "lookup_out.cuh"
#include "trunk.h"

namespace cg {

int forward_ragged_impl(const cg_trunk_dims* dims_p, const void* blob, const float* x_in, const float* ple,
                        const float* values, int64_t batch, int steps, const int64_t* positions,
                        const int64_t* readout_offsets, const int64_t* rows, int span, void* k_pool, void* v_pool,
                        int kv_dtype, int64_t capacity, int max_len, int precision, void* workspace,
                        int64_t workspace_bytes, float* hidden_out, cudaStream_t s, bool x_in_workspace,
                        bool lookup_blocked);
bool tc_layers_available(const cg_trunk_dims& dims);
unsigned char* step_tc_scratch(const cg_trunk_dims& dims, int64_t batch, int steps, int precision, void* workspace);
void tc_input_streams(const cg_trunk_dims& dims, int64_t batch, int steps, unsigned char* scratch, float** x_blk,
                      float** ple_blk, float** val_blk, int64_t* ntiles);

namespace {

constexpr int kBagThreads = 256;

__device__ __forceinline__ int64_t bag_id(const void* ids, int dtype, int64_t index) {
  if (dtype == CG_I16) return static_cast<const int16_t*>(ids)[index];
  if (dtype == CG_I32) return static_cast<const int32_t*>(ids)[index];
  return static_cast<const int64_t*>(ids)[index];
}

template <typename T>
struct BagUnit;  // a 16-byte unit of a table row: load as fp32, store from fp32 (rounded once)

template <>
struct BagUnit<float> {
  static constexpr int kElems = 4;
  static __device__ __forceinline__ void add(const uint4& raw, float (&acc)[4]) {
    acc[0] += __uint_as_float(raw.x);
    acc[1] += __uint_as_float(raw.y);
    acc[2] += __uint_as_float(raw.z);
    acc[3] += __uint_as_float(raw.w);
  }
  static __device__ __forceinline__ void store(void* dst, const float (&acc)[4]) {
    *static_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
};

template <typename H, typename H2>
struct BagUnit16 {
  static constexpr int kElems = 8;
  static __device__ __forceinline__ float2 to_float2(const H2& v);
  static __device__ __forceinline__ void add(const uint4& raw, float (&acc)[8]) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = to_float2(*reinterpret_cast<const H2*>(&w[i]));
      acc[2 * i] += f.x;
      acc[2 * i + 1] += f.y;
    }
  }
};

template <>
struct BagUnit<__nv_bfloat16> : BagUnit16<__nv_bfloat16, __nv_bfloat162> {
  static __device__ __forceinline__ void store(void* dst, const float (&acc)[8]) {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 v = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    *static_cast<uint4*>(dst) = raw;
  }
};
template <>
__device__ __forceinline__ float2 BagUnit16<__nv_bfloat16, __nv_bfloat162>::to_float2(const __nv_bfloat162& v) {
  return __bfloat1622float2(v);
}

template <>
struct BagUnit<__half> : BagUnit16<__half, __half2> {
  static __device__ __forceinline__ void store(void* dst, const float (&acc)[8]) {
    uint4 raw;
    uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __half2 v = __floats2half2_rn(acc[2 * i], acc[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    *static_cast<uint4*>(dst) = raw;
  }
};
template <>
__device__ __forceinline__ float2 BagUnit16<__half, __half2>::to_float2(const __half2& v) {
  return __half22float2(v);
}

struct BagArgs {
  const void* ids;
  int ids_dtype;
  int64_t n, ids_stride;
  int fields;
  int64_t offsets[32];
  const void* table;
  int64_t rows;
  int width;  // elements per row
  void* out;
};

// Resolve this warp's token: lane f < fields holds row ids[f] + offsets[f] if it is in range
// and no lower lane selected the same row. Returns the mask of lanes that contribute.
__device__ __forceinline__ unsigned bag_rows(const BagArgs& a, int64_t token, int lane, int64_t& row) {
  row = -1;
  bool ok = false;
  if (lane < a.fields) {
    const int64_t id = bag_id(a.ids, a.ids_dtype, token * a.ids_stride + lane) + a.offsets[lane];
    if (id < 0 || id >= a.rows) {
      raise_fault(0x210);
    } else {
      row = id;
      ok = true;
    }
  }
  const unsigned live = __ballot_sync(0xffffffffu, ok);
  const unsigned same = __match_any_sync(0xffffffffu, row);
  const bool first = ok && (same & ((1u << lane) - 1u) & live) == 0u;
  return __ballot_sync(0xffffffffu, first);
}

template <typename T>
__global__ void __launch_bounds__(kBagThreads) onehot_bags_kernel(const __grid_constant__ BagArgs a) {
  using U = BagUnit<T>;
  constexpr int kAhead = 8;  // rows whose units are loaded before they are added
  __shared__ const unsigned char* rows_s[kBagThreads / 32][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * kBagThreads + threadIdx.x) >> 5;
  if (token >= a.n) return;
  int64_t row;
  const unsigned keep = bag_rows(a, token, lane, row);
  const int64_t row_bytes = static_cast<int64_t>(a.width) * sizeof(T);
  // Selected rows in field order (ascending lane), each once, as row base addresses.
  if ((keep >> lane) & 1u)
    rows_s[w][__popc(keep & ((1u << lane) - 1u))] = static_cast<const unsigned char*>(a.table) + row * row_bytes;
  __syncwarp();
  const int nk = __popc(keep);
  const int units = a.width / U::kElems;
  unsigned char* out = static_cast<unsigned char*>(a.out) + token * row_bytes;
  for (int u = lane; u < units; u += 32) {
    float acc[U::kElems];
#pragma unroll
    for (int e = 0; e < U::kElems; ++e) acc[e] = 0.f;
    for (int k0 = 0; k0 < nk; k0 += kAhead) {
      uint4 v[kAhead];
#pragma unroll
      for (int i = 0; i < kAhead; ++i)
        if (k0 + i < nk) v[i] = __ldg(reinterpret_cast<const uint4*>(rows_s[w][k0 + i] + 16 * u));
#pragma unroll
      for (int i = 0; i < kAhead; ++i)
        if (k0 + i < nk) U::add(v[i], acc);
    }
    U::store(out + 16 * u, acc);
  }
}

// Any width (not a multiple of the 16-byte unit): one element per lane step.
template <typename T>
__global__ void __launch_bounds__(kBagThreads) onehot_bags_scalar_kernel(const __grid_constant__ BagArgs a) {
  __shared__ int64_t rows_s[kBagThreads / 32][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * kBagThreads + threadIdx.x) >> 5;
  if (token >= a.n) return;
  int64_t row;
  const unsigned keep = bag_rows(a, token, lane, row);
  // Selected rows in field order, each once (the column loop below diverges across lanes,
  // so the rows are read from shared memory, not shuffled).
  if ((keep >> lane) & 1u) rows_s[w][__popc(keep & ((1u << lane) - 1u))] = row;
  __syncwarp();
  const int nk = __popc(keep);
  const T* table = static_cast<const T*>(a.table);
  T* out = static_cast<T*>(a.out) + token * a.width;
  for (int c = lane; c < a.width; c += 32) {
    float acc = 0.f;
    for (int k = 0; k < nk; ++k) acc += static_cast<float>(table[rows_s[w][k] * a.width + c]);
    out[c] = static_cast<T>(acc);
  }
}

// fp32 tables into the trunk's tile-blocked input streams (the first dense kernel conditions
// them), with an optional fp32 addend [n, d] on the x columns (the reference adds the card-grid
// summary to the field sums before Trunk.condition).
__global__ void __launch_bounds__(kBagThreads) onehot_bags_blocked_kernel(const __grid_constant__ BagArgs a,
                                                                           const EmbedOut dest,
                                                                           const float* __restrict__ x_add) {
  constexpr int kAhead = 8;
  __shared__ const unsigned char* rows_s[kBagThreads / 32][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int64_t token = (static_cast<int64_t>(blockIdx.x) * kBagThreads + threadIdx.x) >> 5;
  if (token >= a.n) return;
  int64_t row;
  const unsigned keep = bag_rows(a, token, lane, row);
  const int64_t row_bytes = static_cast<int64_t>(a.width) * 4;
  if ((keep >> lane) & 1u)
    rows_s[w][__popc(keep & ((1u << lane) - 1u))] = static_cast<const unsigned char*>(a.table) + row * row_bytes;
  __syncwarp();
  const int nk = __popc(keep);
  const int units = a.width / 4;
  for (int u = lane; u < units; u += 32) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = 0; k0 < nk; k0 += kAhead) {
      uint4 v[kAhead];
#pragma unroll
      for (int i = 0; i < kAhead; ++i)
        if (k0 + i < nk) v[i] = __ldg(reinterpret_cast<const uint4*>(rows_s[w][k0 + i] + 16 * u));
#pragma unroll
      for (int i = 0; i < kAhead; ++i)
        if (k0 + i < nk) BagUnit<float>::add(v[i], acc);
    }
    if (x_add && 4 * u < dest.d) {
      const float4 e = __ldg(reinterpret_cast<const float4*>(x_add + token * dest.d) + u);
      acc[0] += e.x;
      acc[1] += e.y;
      acc[2] += e.z;
      acc[3] += e.w;
    }
    const LookupColumn col = lookup_column(dest, u);
    col.base[(token >> 7) * col.tile_stride + (token & 127)] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  }
}

template <typename T>
int launch_bags(const BagArgs& a, cudaStream_t s) {
  const unsigned blocks = static_cast<unsigned>((a.n * 32 + kBagThreads - 1) / kBagThreads);
  const bool vec = (static_cast<int64_t>(a.width) * sizeof(T)) % 16 == 0 &&
                   (reinterpret_cast<uintptr_t>(a.table) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
  if (vec) {
    onehot_bags_kernel<T><<<blocks, kBagThreads, 0, s>>>(a);
    return check_launch("onehot_bags_kernel");
  }
  onehot_bags_scalar_kernel<T><<<blocks, kBagThreads, 0, s>>>(a);
  return check_launch("onehot_bags_scalar_kernel");
}

}  // namespace
}  // namespace cg

extern "C" int cg_onehot_bags(const void* ids, int ids_dtype, int64_t n_tokens, int64_t ids_stride, int fields,
                              const int64_t* offsets, const void* table, int table_dtype, int64_t rows, int width,
                              void* out, void* stream) {
  using namespace cg;
  CG_REQUIRE(ids_dtype == CG_I16 || ids_dtype == CG_I32 || ids_dtype == CG_I64, "cg_onehot_bags: bad id dtype");
  CG_REQUIRE(table_dtype == CG_F32 || table_dtype == CG_BF16 || table_dtype == CG_F16,
             "cg_onehot_bags: bad table dtype");
  CG_REQUIRE(fields >= 1 && fields <= 32, "cg_onehot_bags: fields must be 1..32 (got %d)", fields);
  CG_REQUIRE(n_tokens >= 0 && rows >= 1 && width >= 1, "cg_onehot_bags: bad sizes");
  CG_REQUIRE(ids_stride >= fields, "cg_onehot_bags: id row stride %lld < %d fields", (long long)ids_stride, fields);
  if (n_tokens == 0) return CG_OK;
  CG_REQUIRE(ids && table && out, "cg_onehot_bags: NULL pointer");
  CG_REQUIRE(n_tokens <= (int64_t(1) << 40), "cg_onehot_bags: too many tokens");
  BagArgs a{};
  a.ids = ids;
  a.ids_dtype = ids_dtype;
  a.n = n_tokens;
  a.ids_stride = ids_stride;
  a.fields = fields;
  for (int f = 0; f < fields; ++f) a.offsets[f] = offsets ? offsets[f] : 0;
  a.table = table;
  a.rows = rows;
  a.width = width;
  a.out = out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (table_dtype == CG_F32) return launch_bags<float>(a, s);
  if (table_dtype == CG_BF16) return launch_bags<__nv_bfloat16>(a, s);
  return launch_bags<__half>(a, s);
}

extern "C" int cg_bags_forward_ragged(const cg_trunk_dims* dims, const void* blob, const void* ids, int ids_dtype,
                                      int64_t ids_stride, int fields, const int64_t* offsets, const float* table,
                                      int64_t table_rows, const float* x_add, int64_t batch, int steps,
                                      const int64_t* positions, const int64_t* readout_offsets, const int64_t* rows,
                                      int span, void* k_pool, void* v_pool, int kv_dtype, int64_t capacity,
                                      int max_len, int precision, void* workspace, int64_t workspace_bytes,
                                      float* hidden_out, void* stream) {
  using namespace cg;
  CG_REQUIRE(dims, "cg_bags_forward_ragged: NULL trunk dims");
  CG_REQUIRE(precision == CG_PREC_BF16 && tc_layers_available(*dims),
             "cg_bags_forward_ragged: the fused lookup feeds the tensor-core layers (bf16 precision) only");
  CG_REQUIRE(ids_dtype == CG_I16 || ids_dtype == CG_I32 || ids_dtype == CG_I64, "cg_bags_forward_ragged: bad id dtype");
  CG_REQUIRE(fields >= 1 && fields <= 32, "cg_bags_forward_ragged: fields must be 1..32 (got %d)", fields);
  CG_REQUIRE(ids_stride >= fields && table_rows >= 1, "cg_bags_forward_ragged: bad id stride or table");
  if (batch == 0) return CG_OK;
  CG_REQUIRE(ids && table && workspace && blob, "cg_bags_forward_ragged: NULL pointer");
  CG_REQUIRE((reinterpret_cast<uintptr_t>(table) & 15) == 0 && (reinterpret_cast<uintptr_t>(x_add) & 15) == 0,
             "cg_bags_forward_ragged: table and x_add must be 16-byte aligned");
  const int64_t need = cg_trunk_step_workspace_bytes(dims, batch, steps, precision);
  if (need < 0) return set_error(CG_ERR_ARGUMENT, "cg_bags_forward_ragged: bad trunk dims");
  if (workspace_bytes < need)
    return set_error(CG_ERR_WORKSPACE, "bags step workspace %lld < %lld bytes", (long long)workspace_bytes,
                     (long long)need);
  const cg_trunk_dims& d = *dims;
  EmbedOut dest{};
  dest.d = d.d_model;
  dest.ple_w = d.n_layers * d.per_layer_dim;
  dest.P = d.per_layer_dim;
  dest.kvw = d.n_kv_heads * head_dim(d);
  const int width = dest.d + dest.ple_w + value_layer_count(d) * dest.kvw;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  tc_input_streams(d, batch, steps, step_tc_scratch(d, batch, steps, precision, workspace), &dest.x_blk, &dest.ple_blk,
                   &dest.val_blk, &dest.ntiles);
  BagArgs a{};
  a.ids = ids;
  a.ids_dtype = ids_dtype;
  a.n = batch * steps;
  a.ids_stride = ids_stride;
  a.fields = fields;
  for (int f = 0; f < fields; ++f) a.offsets[f] = offsets ? offsets[f] : 0;
  a.table = table;
  a.rows = table_rows;
  a.width = width;
  const unsigned blocks = static_cast<unsigned>((a.n * 32 + kBagThreads - 1) / kBagThreads);
  onehot_bags_blocked_kernel<<<blocks, kBagThreads, 0, s>>>(a, dest, x_add);
  int rc;
  if ((rc = check_launch("onehot_bags_blocked_kernel"))) return rc;
  return forward_ragged_impl(dims, blob, nullptr, nullptr, nullptr, batch, steps, positions, readout_offsets, rows,
                             span, k_pool, v_pool, kv_dtype, capacity, max_len, precision, workspace, workspace_bytes,
                             hidden_out, s, false, true);
}
