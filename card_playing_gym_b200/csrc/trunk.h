// Internal interfaces shared by the trunk translation units.
#pragma once

#include "common.cuh"

namespace cg {

struct AttnParams {
  const void* q;
  int q_dtype;
  int64_t q_sb, q_sh, q_st;  // q strides (elements) over batch, head, step; d is contiguous
  const void* k;
  const void* v;
  int kv_dtype;
  int64_t kv_row, kv_head, kv_pos;  // cache strides (elements); d contiguous
  const int64_t* rows;
  const int64_t* lengths;
  int64_t batch;
  int heads, kv_heads, steps, group, head_dim, span;
  float scale;
  void* out;
  int out_dtype;
  int64_t o_sb, o_sh, o_st;
  // out_blocked: write the output as the next GEMM's operand, tile-blocked bf16: element
  // (row-token r = b*T + t, column k = h*D + d) at ((r/128) * W/8 + k/8) * 1024 + (r%128) * 8 + k%8,
  // W = blocked_width (= heads * head_dim).
  int out_blocked;
  int blocked_width;
  // Dynamic work distribution: warps claim (row, KV head) units from this counter, which
  // must be zero at launch (nullptr: a static stride over the units).
  int* counter;
};

__host__ __device__ inline int64_t blocked_offset(int64_t r, int k, int width) {
  return ((r / 128) * (width / 8) + k / 8) * 1024 + (r % 128) * 8 + (k % 8);
}

int run_attention(const AttnParams& p, cudaStream_t stream);

// Byte layout of the trunk weight blob. The fp32 section mirrors the reference's
// parameters; the bf16 section holds the tensor-core operand copies of the five
// GEMM weight kinds (ple_context, qkv, out, up, down) in the layout tc_pack writes.
struct BlobLayout {
  int64_t fp32[CG_PART_COUNT];      // trunk-wide parts (layer-independent), byte offsets or -1
  int64_t layer_base;               // byte offset of layer 0's per-layer block
  int64_t layer_stride;             // bytes per layer block
  int64_t layer_part[CG_PART_COUNT];  // byte offset within a layer block, or -1
  int64_t bf16_ple_context;         // byte offsets of the bf16 copies
  int64_t bf16_layer_base, bf16_layer_stride;
  int64_t bf16_qkv, bf16_out, bf16_up, bf16_down;  // within a bf16 layer block
  int64_t total;
};

BlobLayout blob_layout(const cg_trunk_dims& dims);

inline int qkv_width(const cg_trunk_dims& d) { return (d.n_heads + 2 * d.n_kv_heads) * (d.d_model / d.n_heads); }
inline int head_dim(const cg_trunk_dims& d) { return d.d_model / d.n_heads; }
inline int value_layer_count(const cg_trunk_dims& d) {
  int n = 0;
  for (int l = 0; l < d.n_layers; ++l) n += (d.value_layers >> l) & 1;
  return n;
}
inline int value_index(const cg_trunk_dims& d, int layer) {
  if (!((d.value_layers >> layer) & 1)) return -1;
  int n = 0;
  for (int l = 0; l < layer; ++l) n += (d.value_layers >> l) & 1;
  return n;
}

template <typename T>
inline const T* blob_ptr(const void* blob, int64_t offset) {
  return reinterpret_cast<const T*>(static_cast<const unsigned char*>(blob) + offset);
}

inline const float* part(const void* blob, const BlobLayout& L, int which, int layer) {
  if (which <= CG_PART_FINAL_B) return L.fp32[which] < 0 ? nullptr : blob_ptr<float>(blob, L.fp32[which]);
  return blob_ptr<float>(blob, L.layer_base + layer * L.layer_stride + L.layer_part[which]);
}

}  // namespace cg
