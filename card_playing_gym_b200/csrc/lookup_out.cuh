// Where a field lookup writes its sums: row-major, or straight into the first dense kernel's
// tile-blocked input streams. Shared by the plump lookup (plump.cu) and the one-hot field
// bags (bags.cu).
#pragma once

#include "common.cuh"

namespace cg {

// Destination of the lookup sums: row-major [n, width], or the trunk's tile-blocked streams
// (x_blk non-null): columns [0, d) -> x_blk, [d, d + L*P) -> ple_blk (per layer), the rest ->
// val_blk (per value layer), each [.. tile][width/4][128 rows][4].
struct EmbedOut {
  float* rows;
  float* x_blk;
  float* ple_blk;
  float* val_blk;
  int d, ple_w, P, kvw;
  int64_t ntiles;
};

// Blocked destination of float4 column c4 for tile 0, row 0, and the step from one tile to the
// next: the token-independent part of a sum's blocked address, computed once per column.
struct LookupColumn {
  float4* base;
  int64_t tile_stride;
};

__device__ __forceinline__ LookupColumn lookup_column(const EmbedOut& o, int c4) {
  int k = 4 * c4;
  if (k < o.d) return {reinterpret_cast<float4*>(o.x_blk) + static_cast<int64_t>(k / 4) * 128, (o.d / 4) * 128};
  if ((k -= o.d) < o.ple_w) {
    const int layer = k / o.P, q = k - layer * o.P;
    return {reinterpret_cast<float4*>(o.ple_blk) + (layer * o.ntiles * (o.P / 4) + q / 4) * 128, (o.P / 4) * 128};
  }
  k -= o.ple_w;
  const int vl = k / o.kvw, q = k - vl * o.kvw;
  return {reinterpret_cast<float4*>(o.val_blk) + (vl * o.ntiles * (o.kvw / 4) + q / 4) * 128, (o.kvw / 4) * 128};
}

}  // namespace cg
