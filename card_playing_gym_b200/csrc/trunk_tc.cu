// Tensor-core (tcgen05) dense layers of the bf16 decode step.
//
// This unit owns the bf16 section of the trunk weight blob: tc_pack writes the
// bf16 operand copies of ple_context, qkv, out, up and down there.
#include "trunk.h"

namespace cg {

int64_t tc_pack_bytes_ple(const cg_trunk_dims& dims) {
  return static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim * dims.d_model * 2;
}

int64_t tc_pack_bytes_layer(const cg_trunk_dims& dims) {
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  return (q * d + d * d + f * d + d * f) * 2 + 4 * 256;
}

__global__ void tc_pack_copy_kernel(const float* in, __nv_bfloat16* out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = __float2bfloat16_rn(in[i]);
}

int tc_pack(const cg_trunk_dims& dims, void* blob, const BlobLayout& L, cudaStream_t s) {
  unsigned char* base = static_cast<unsigned char*>(blob);
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  auto copy = [&](const float* src, int64_t dst_off, int64_t n) {
    tc_pack_copy_kernel<<<static_cast<unsigned>((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, s>>>(
        src, reinterpret_cast<__nv_bfloat16*>(base + dst_off), n);
    return check_launch("tc_pack_copy_kernel");
  };
  int rc;
  if (dims.per_layer_dim) {
    if ((rc = copy(part(blob, L, CG_PART_PLE_CONTEXT, 0), L.bf16_ple_context, tc_pack_bytes_ple(dims) / 2))) return rc;
  }
  for (int layer = 0; layer < dims.n_layers; ++layer) {
    int64_t at = L.bf16_layer_base + layer * L.bf16_layer_stride;
    if ((rc = copy(part(blob, L, CG_PART_QKV, layer), at, q * d))) return rc;
    at += (q * d * 2 + 255) / 256 * 256;
    if ((rc = copy(part(blob, L, CG_PART_OUT, layer), at, d * d))) return rc;
    at += (d * d * 2 + 255) / 256 * 256;
    if ((rc = copy(part(blob, L, CG_PART_UP, layer), at, f * d))) return rc;
    at += (f * d * 2 + 255) / 256 * 256;
    if ((rc = copy(part(blob, L, CG_PART_DOWN, layer), at, d * f))) return rc;
  }
  return CG_OK;
}

bool tc_layers_available(const cg_trunk_dims&) { return false; }

int64_t tc_layers_scratch_bytes(const cg_trunk_dims&, int64_t, int) { return 0; }

int run_tc_layers(const cg_trunk_dims&, const void*, const BlobLayout&, int64_t, int, const int64_t*, const int64_t*,
                  const int64_t*, int, void*, void*, int, int64_t, int, float*, const float*, const float*,
                  unsigned char*, int64_t, cudaStream_t) {
  return set_error(CG_ERR_ARGUMENT, "tensor-core dense layers are not available for these dims");
}

int tc_condition_ple(const cg_trunk_dims&, const void*, const BlobLayout&, const float*, const float*, int64_t, int64_t,
                     float*, cudaStream_t) {
  return set_error(CG_ERR_ARGUMENT, "tensor-core conditioning is not available for these dims");
}

}  // namespace cg
