// Tensor-core (tcgen05) dense layers of the bf16 ragged decode step.
//
// Reference arithmetic: cardgym/nn/trunk.py — condition 285-312 (RMSNorm, PLE context
// projection), DecoderBlock._qkv 141-152 (LN, fused QKV, value embedding),
// _finish 154-157 (out projection + residual, LN, GELU MLP + residual), _add_ple
// 318-333, and the KV append of kv_cache.py:84-105 with trunk.py:419-423's clamp.
//
// One CTA owns a tile of 128 row-tokens and carries it across a layer boundary:
//   attention(l) output -> out_proj -> x += . -> LN -> up (d-wide chunks) -> GELU ->
//   down (accumulated over the chunks) -> x += . + b -> x += PLE(l) -> LN -> QKV(l+1)
//   -> q for attention(l+1), K/V appended to the pool.
// Roles: warps 0-3 are epilogue warps (thread t owns row t = TMEM lane t); warp 4's
// lane 0 streams weight K-slices into a ring of shared-memory stages with bulk async
// copies; warp 5 allocates tensor memory and its lane 0 issues tcgen05.mma (M=128,
// bf16 x bf16 -> fp32 in TMEM). The GEMM weights are pre-packed (tc_pack) so each
// K=16 slice is one contiguous bulk copy already in the canonical operand layout.
//
// Activations between kernels live in a tile-blocked layout so that thread-per-row
// access is coalesced: element (row r, column k) of an fp32 [rows, width] array sits
// at float4 index ((tile * width/4 + k/4) * 128 + r % 128), lane k % 4; the
// attention output (the out-projection operand) is bf16 in the operand layout itself:
// tile block = width/8 chunks of [128 rows x 8 columns].
#include <cmath>

#include "tcgen05.cuh"
#include "trunk.h"

namespace cg {

constexpr int kTile = 128;
constexpr int kTcThreads = 192;
constexpr int kMaxOps = 16;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 225 * 1024;

enum TcMode { kLayer = 0, kFirstLookup = 1, kFirstConditioned = 2 };

struct GemmOp {
  const __nv_bfloat16* w;  // packed K-slices: ksteps x [n rows x 16 columns]
  int n;
  int ksteps;
  int tmem_col;
  int a_src;  // 0: A buffer, 1: H buffer
  int accumulate_first;
  int wait_a;
  int signal;
};

struct TcParams {
  int mode, layer, qkv_layer, has_next;
  GemmOp ops[kMaxOps];
  int n_ops, stages, stage_bytes;
  int d, f, H, KVH, D, L, P, nv, kvw, qw;
  int64_t nt, ntiles;
  int T;
  float* x_blk;
  float* ple_blk;
  float* val_blk;
  const __nv_bfloat16* attn_blk;
  void* q;
  int q_dtype;
  const float* lookup;  // kFirstLookup: raw lookup rows [nt, lookup_width]
  int lookup_width;
  const float* x_in;  // kFirstConditioned inputs
  const float* ple_in;
  const float* val_in;
  const float* rms_w;
  const float* ln_mlp_w;
  const float* ln_mlp_b;
  const float* up_b;
  const float* down_b;
  const float* ln_next_w;
  const float* ln_next_b;
  float ple_scale;
  int value_index;  // value-embedding index of qkv_layer, -1: none
  void* k_layer;
  void* v_layer;
  int kv_dtype, max_len;
  const int64_t* positions;
  const int64_t* rows;
};

// ---- blocked activation helpers -------------------------------------------------------------
__device__ __forceinline__ float4* blk(float* base, int64_t tile, int width, int k, int t) {
  return reinterpret_cast<float4*>(base) + ((tile * (width / 4) + k / 4) * kTile + t);
}

__device__ __forceinline__ void load16(const float* base, int64_t tile, int width, int col, int t, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = *blk(const_cast<float*>(base), tile, width, col + 4 * q, t);
    v[4 * q] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
}

__device__ __forceinline__ void store16(float* base, int64_t tile, int width, int col, int t, const float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *blk(base, tile, width, col + 4 * q, t) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// 16 consecutive columns (col % 16 == 0) of row t as bf16 into the operand layout.
__device__ __forceinline__ void store_operand16(unsigned char* buf, int col, int t, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint4 packed;
    uint32_t* words = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 pair = __floats2bfloat162_rn(v[8 * h + 2 * i], v[8 * h + 2 * i + 1]);
      words[i] = *reinterpret_cast<uint32_t*>(&pair);
    }
    *reinterpret_cast<uint4*>(buf + (col / 8 + h) * (kTile * 16) + t * 16) = packed;
  }
}

// LayerNorm (eps 1e-5, biased variance, two passes) of row t of the blocked x into the A buffer.
__device__ void layer_norm_to_operand(const float* x, int64_t tile, int d, int t, const float* w, const float* b,
                                      unsigned char* abuf) {
  float v[16];
  float sum = 0.f;
  for (int col = 0; col < d; col += 16) {
    load16(x, tile, d, col, t, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) sum += v[i];
  }
  const float mean = sum / d;
  float var = 0.f;
  for (int col = 0; col < d; col += 16) {
    load16(x, tile, d, col, t, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float c = v[i] - mean;
      var += c * c;
    }
  }
  const float rstd = rsqrtf(var / d + 1e-5f);
  for (int col = 0; col < d; col += 16) {
    load16(x, tile, d, col, t, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = (v[i] - mean) * rstd * w[col + i] + b[col + i];
    store_operand16(abuf, col, t, v);
  }
}

// ---- the QKV epilogue: q out, K/V (+ value embedding) into the pool ------------------------------------
__device__ void qkv_epilogue(const TcParams& p, uint32_t lane_tmem, int64_t tile, int t) {
  const int64_t row = tile * kTile + t;
  const bool valid = row < p.nt;
  const int64_t b = row / p.T;
  const int tt = static_cast<int>(row % p.T);
  int64_t pos = 0, cache_row = 0;
  if (valid) {
    pos = p.positions[b] + tt;
    if (pos > p.max_len - 1) pos = p.max_len - 1;
    cache_row = p.rows ? p.rows[b] : b;
  }
  const int hd = p.H * p.D;
  float v[16];
  for (int col0 = 0; col0 < p.qw; col0 += 16) {
    tc::tmem_ld16(lane_tmem + col0, v);
    if (!valid) continue;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int col = col0 + i;
      if (col < hd) {
        const int h = col / p.D, dd = col % p.D;
        store_from_float(p.q, ((b * p.H + h) * p.T + tt) * p.D + dd, p.q_dtype, v[i]);
      } else {
        const int cc = col - hd;
        const int which = cc / p.kvw, rem = cc % p.kvw;
        const int kvh = rem / p.D, dd = rem % p.D;
        float value = v[i];
        if (which == 1 && p.value_index >= 0) {
          const float4 e = *blk(p.val_blk, static_cast<int64_t>(p.value_index) * p.ntiles + tile, p.kvw, rem, t);
          const int lanei = rem & 3;
          value += lanei == 0 ? e.x : lanei == 1 ? e.y : lanei == 2 ? e.z : e.w;
        }
        const int64_t dst = ((cache_row * p.KVH + kvh) * p.max_len + pos) * p.D + dd;
        store_from_float(which ? p.v_layer : p.k_layer, dst, p.kv_dtype, value);
      }
    }
  }
}

// ---- epilogue warps (threads 0..127: thread t owns row t of the tile and TMEM lane t) ----------------
__device__ void dense_epilogue(const TcParams& p, unsigned char* abuf, unsigned char* hbuf, uint32_t tmem,
                               uint64_t* a_ready_bar, uint64_t* acc_ready_bar, uint64_t* attn_full_bar, int abytes) {
  const int warp = threadIdx.x >> 5;
  const int64_t tile = blockIdx.x;
  uint64_t& a_ready = *a_ready_bar;
  uint64_t& acc_ready = *acc_ready_bar;
  uint64_t& attn_full = *attn_full_bar;
    const int t = threadIdx.x;  // row within the tile == TMEM lane
    const uint32_t lane_tmem = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int64_t row = tile * kTile + t;
    const bool valid = row < p.nt;
    uint32_t acc_phase = 0;
    float v[16], x[16];
    const int d = p.d;
    auto publish = [&]() {  // operand written and TMEM reads done: hand over to the MMA warp
      tc::fence_async_smem();
      tc::fence_before_sync();
      tc::bar_arrive(&a_ready);
    };
    auto wait_acc = [&]() -> bool {
      if (!tc::bar_wait(&acc_ready, acc_phase, 0x403)) return false;
      acc_phase ^= 1u;
      tc::fence_after_sync();
      return true;
    };

    if (p.mode == kLayer) {
      // E0: the attention output tile is already in operand layout: one bulk copy.
      if (t == 0) {
        tc::bar_expect_tx(&attn_full, abytes);
        tc::bulk_g2s(abuf, reinterpret_cast<const unsigned char*>(p.attn_blk) + tile * abytes, abytes, &attn_full);
      }
      if (!tc::bar_wait(&attn_full, 0, 0x404)) return;
      publish();
      // E1: x += out_proj; LN_mlp(x) -> A.
      if (!wait_acc()) return;
      for (int col = 0; col < d; col += 16) {
        tc::tmem_ld16(lane_tmem + p.ops[0].tmem_col + col, v);
        load16(p.x_blk, tile, d, col, t, x);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] += v[i];
        store16(p.x_blk, tile, d, col, t, x);
      }
      layer_norm_to_operand(p.x_blk, tile, d, t, p.ln_mlp_w, p.ln_mlp_b, abuf);
      publish();
      // E2: GELU of each up chunk into H.
      const int chunks = p.f / d;
      for (int c = 0; c < chunks; ++c) {
        if (!wait_acc()) return;
        for (int col = 0; col < d; col += 16) {
          tc::tmem_ld16(lane_tmem + 256 + col, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = gelu_erf(v[i] + p.up_b[c * d + col + i]);
          store_operand16(hbuf, col, t, v);
        }
        publish();
      }
      // E3: x += down + b; x += PLE(l); then LN_attn(l+1) -> A.
      if (!wait_acc()) return;
      for (int col = 0; col < d; col += 16) {
        tc::tmem_ld16(lane_tmem + col, v);
        load16(p.x_blk, tile, d, col, t, x);
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] += v[i] + p.down_b[col + i];
        if (p.P) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const int k = (col + i) % p.P;  // P % 4 == 0: four columns share a float4
            const float4 e = *blk(p.ple_blk, static_cast<int64_t>(p.layer) * p.ntiles + tile, p.P, k, t);
            x[i] += e.x * p.ple_scale;
            x[i + 1] += e.y * p.ple_scale;
            x[i + 2] += e.z * p.ple_scale;
            x[i + 3] += e.w * p.ple_scale;
          }
        }
        store16(p.x_blk, tile, d, col, t, x);
      }
      if (p.has_next) {
        layer_norm_to_operand(p.x_blk, tile, d, t, p.ln_next_w, p.ln_next_b, abuf);
        publish();
        if (!wait_acc()) return;
        qkv_epilogue(p, lane_tmem, tile, t);
      }
    } else {
      // First kernel of a wave: conditioned x, PLE and value streams into blocked layout.
      const int ple_w = p.L * p.P;
      const int val_w = p.nv * p.kvw;
      const float inv_sqrt2 = 0.70710678118654752f;
      if (p.mode == kFirstLookup) {
        const float* src = p.lookup + (valid ? row : 0) * p.lookup_width;
        // x = RMSNorm(lookup[:, :d]) * gain (trunk.py:297-298, 104-115)
        float ss = 0.f;
        for (int col = 0; col < d; col += 4) {
          const float4 e = *reinterpret_cast<const float4*>(src + col);
          ss += e.x * e.x + e.y * e.y + e.z * e.z + e.w * e.w;
        }
        const float inv = rsqrtf(ss / d + 1e-5f);
        for (int col = 0; col < d; col += 16) {
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 e = *reinterpret_cast<const float4*>(src + col + i);
            x[i] = e.x * inv * p.rms_w[col + i];
            x[i + 1] = e.y * inv * p.rms_w[col + i + 1];
            x[i + 2] = e.z * inv * p.rms_w[col + i + 2];
            x[i + 3] = e.w * inv * p.rms_w[col + i + 3];
          }
          store16(p.x_blk, tile, d, col, t, x);
          store_operand16(abuf, col, t, x);
        }
        for (int c4 = 0; c4 < val_w; c4 += 4) {
          const float4 e = *reinterpret_cast<const float4*>(src + d + ple_w + c4);
          *blk(p.val_blk, static_cast<int64_t>(c4 / p.kvw) * p.ntiles + tile, p.kvw, c4 % p.kvw, t) = e;
        }
        if (p.n_ops > 1) publish();
        // ple = (lookup + W_c x) / sqrt(2), one TMEM chunk of up to 256 columns at a time.
        int c0 = 0;
        for (int o = 0; o + 1 < p.n_ops; ++o) {
          const int n = p.ops[o].n;
          if (!wait_acc()) return;
          for (int col = 0; col < n; col += 16) {
            tc::tmem_ld16(lane_tmem + col, v);
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const int k = c0 + col + i;
              const float4 e = *reinterpret_cast<const float4*>(src + d + k);
              const int layer = k / p.P, kk = k % p.P;
              *blk(p.ple_blk, static_cast<int64_t>(layer) * p.ntiles + tile, p.P, kk, t) =
                  make_float4((e.x + v[i]) * inv_sqrt2, (e.y + v[i + 1]) * inv_sqrt2, (e.z + v[i + 2]) * inv_sqrt2,
                              (e.w + v[i + 3]) * inv_sqrt2);
            }
          }
          c0 += n;
          if (o + 2 < p.n_ops) publish();
        }
      } else {
        const int64_t r = valid ? row : 0;
        for (int col = 0; col < d; col += 16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) x[i] = p.x_in[r * d + col + i];
          store16(p.x_blk, tile, d, col, t, x);
        }
        for (int k = 0; k < ple_w; k += 4) {
          const float4 e = *reinterpret_cast<const float4*>(p.ple_in + r * ple_w + k);
          *blk(p.ple_blk, static_cast<int64_t>(k / p.P) * p.ntiles + tile, p.P, k % p.P, t) = e;
        }
        for (int k = 0; k < val_w; k += 4) {
          const float4 e = *reinterpret_cast<const float4*>(p.val_in + r * val_w + k);
          *blk(p.val_blk, static_cast<int64_t>(k / p.kvw) * p.ntiles + tile, p.kvw, k % p.kvw, t) = e;
        }
      }
      (void)ple_w;
      layer_norm_to_operand(p.x_blk, tile, d, t, p.ln_next_w, p.ln_next_b, abuf);
      publish();
      if (!wait_acc()) return;
      qkv_epilogue(p, lane_tmem, tile, t);
    }
  }

// ---- the kernel ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kTcThreads, 1) tc_dense_kernel(const __grid_constant__ TcParams p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
  __shared__ __align__(8) uint64_t a_ready, acc_ready, attn_full;
  __shared__ uint32_t tmem_base;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  const int abytes = kTile * p.d * 2;
  unsigned char* abuf = smem;
  unsigned char* hbuf = smem + abytes;
  unsigned char* ring = smem + 2 * abytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      tc::bar_init(&full[s], 1);
      tc::bar_init(&empty[s], 1);
    }
    tc::bar_init(&a_ready, 4 * 32);
    tc::bar_init(&acc_ready, 1);
    tc::bar_init(&attn_full, 1);
    tc::bar_fence_init();
  }
  if (warp == 5) {
    tc::tmem_alloc(&tmem_base, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base;

  if (warp == 4) {
    // ---- producer: weight K-slices into the ring -------------------------------------------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int o = 0; o < p.n_ops && ok; ++o) {
        const GemmOp& op = p.ops[o];
        const uint32_t bytes = static_cast<uint32_t>(op.n) * 32u;
        for (int s = 0; s < op.ksteps; ++s, ++it) {
          const int stage = it % p.stages;
          const int fill = it / p.stages;
          if (fill > 0 && !(ok = tc::bar_wait(&empty[stage], (fill - 1) & 1, 0x400))) break;
          tc::bar_expect_tx(&full[stage], bytes);
          tc::bulk_g2s(ring + stage * p.stage_bytes, op.w + static_cast<int64_t>(s) * op.n * 16, bytes, &full[stage]);
        }
      }
    }
  } else if (warp == 5) {
    // ---- MMA issuer ---------------------------------------------------------------------------------
    if (lane == 0) {
      int it = 0;
      uint32_t a_phase = 0;
      bool ok = true;
      for (int o = 0; o < p.n_ops && ok; ++o) {
        const GemmOp& op = p.ops[o];
        if (op.wait_a) {
          if (!(ok = tc::bar_wait(&a_ready, a_phase, 0x401))) break;
          a_phase ^= 1u;
          tc::fence_after_sync();
        }
        const unsigned char* a_base = op.a_src ? hbuf : abuf;
        for (int s = 0; s < op.ksteps; ++s, ++it) {
          const int stage = it % p.stages;
          if (!(ok = tc::bar_wait(&full[stage], (it / p.stages) & 1, 0x402))) break;
          tc::fence_after_sync();
          const uint64_t a_desc = tc::smem_desc(tc::smem_u32(a_base + 2 * s * (kTile * 16)), kTile * 16, 128);
          const uint32_t b_addr = tc::smem_u32(ring + stage * p.stage_bytes);
          const uint32_t acc = (s > 0 || op.accumulate_first) ? 1u : 0u;
          if (op.n <= 256) {
            tc::mma_bf16(tmem + op.tmem_col, a_desc, tc::smem_desc(b_addr, 128, 256), tc::idesc_bf16(128, op.n), acc);
          } else {
            tc::mma_bf16(tmem + op.tmem_col, a_desc, tc::smem_desc(b_addr, 128, 256), tc::idesc_bf16(128, 256), acc);
            tc::mma_bf16(tmem + op.tmem_col + 256, a_desc, tc::smem_desc(b_addr + 32 * 256, 128, 256),
                         tc::idesc_bf16(128, op.n - 256), acc);
          }
          tc::mma_commit(&empty[stage]);
        }
        if (ok && op.signal) tc::mma_commit(&acc_ready);
      }
    }
  } else {
    dense_epilogue(p, abuf, hbuf, tmem, &a_ready, &acc_ready, &attn_full, abytes);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ---- weight packing --------------------------------------------------------------------------------------
// dst slices s = 0..K/16-1, each [N rows x 16 columns] as core matrices (group g, half h) at (2g + h) * 64 elements.
__global__ void pack_kernel(const float* __restrict__ w, int ldw, int n0, int N, int k0, int K,
                            __nv_bfloat16* __restrict__ dst) {
  const int64_t total = static_cast<int64_t>(N) * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i % 8);
    const int r = static_cast<int>((i / 8) % 8);
    const int h = static_cast<int>((i / 64) % 2);
    const int g = static_cast<int>((i / 128) % (N / 8));
    const int s = static_cast<int>(i / (static_cast<int64_t>(N) * 16));
    const float value = w[static_cast<int64_t>(n0 + g * 8 + r) * ldw + k0 + s * 16 + h * 8 + e];
    dst[i] = __float2bfloat16_rn(value);
  }
}

int64_t tc_pack_bytes_ple(const cg_trunk_dims& dims) {
  return static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim * dims.d_model * 2;
}

int64_t tc_pack_bytes_layer(const cg_trunk_dims& dims) {
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  return (q * d + d * d + 2 * f * d) * 2;
}

struct LayerPack {
  const __nv_bfloat16* qkv;
  const __nv_bfloat16* out;
  const __nv_bfloat16* up;    // chunk c at c * d * d
  const __nv_bfloat16* down;  // chunk c at c * d * d
};

LayerPack layer_pack(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int layer) {
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  const __nv_bfloat16* base = blob_ptr<__nv_bfloat16>(blob, L.bf16_layer_base + layer * L.bf16_layer_stride);
  return {base, base + q * d, base + q * d + d * d, base + q * d + d * d + f * d};
}

bool tc_layers_available(const cg_trunk_dims& dims) {
  const int d = dims.d_model, D = head_dim(dims), q = qkv_width(dims);
  if (d % 16 || d > 256 || dims.d_ff % d || q % 16 || q > 512 || D % 8) return false;
  if (q > 256 && (q - 256) % 16) return false;
  if (dims.per_layer_dim % 4 || (static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim) % 16) return false;
  if ((dims.n_kv_heads * D) % 4) return false;
  const int64_t abytes = static_cast<int64_t>(kTile) * d * 2;
  const int64_t stage = 32LL * (q > 256 ? q : 256);
  return 2 * abytes + 2 * stage <= kSmemBudget;
}

int tc_pack(const cg_trunk_dims& dims, void* blob, const BlobLayout& L, cudaStream_t s) {
  const int d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  auto pack = [&](const float* w, int ldw, int n0, int N, int k0, int K, __nv_bfloat16* dst) {
    const int64_t total = static_cast<int64_t>(N) * K;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    pack_kernel<<<blocks, 256, 0, s>>>(w, ldw, n0, N, k0, K, dst);
    return check_launch("pack_kernel");
  };
  if (!tc_layers_available(dims)) return CG_OK;  // the fp32 copies serve the CUDA-core path
  int rc;
  unsigned char* base = static_cast<unsigned char*>(blob);
  const int ple_w = dims.n_layers * dims.per_layer_dim;
  for (int c0 = 0; c0 < ple_w; c0 += 256) {
    const int n = ple_w - c0 < 256 ? ple_w - c0 : 256;
    auto* dst = reinterpret_cast<__nv_bfloat16*>(base + L.bf16_ple_context) + static_cast<int64_t>(c0) * d;
    if ((rc = pack(part(blob, L, CG_PART_PLE_CONTEXT, 0), d, c0, n, 0, d, dst))) return rc;
  }
  for (int layer = 0; layer < dims.n_layers; ++layer) {
    LayerPack lp = layer_pack(dims, blob, L, layer);
    if ((rc = pack(part(blob, L, CG_PART_QKV, layer), d, 0, q, 0, d, const_cast<__nv_bfloat16*>(lp.qkv)))) return rc;
    if ((rc = pack(part(blob, L, CG_PART_OUT, layer), d, 0, d, 0, d, const_cast<__nv_bfloat16*>(lp.out)))) return rc;
    for (int c = 0; c < f / d; ++c) {
      if ((rc = pack(part(blob, L, CG_PART_UP, layer), d, c * d, d, 0, d,
                     const_cast<__nv_bfloat16*>(lp.up) + static_cast<int64_t>(c) * d * d)))
        return rc;
      if ((rc = pack(part(blob, L, CG_PART_DOWN, layer), f, 0, d, c * d, d,
                     const_cast<__nv_bfloat16*>(lp.down) + static_cast<int64_t>(c) * d * d)))
        return rc;
    }
  }
  return CG_OK;
}

// ---- scratch and orchestration ------------------------------------------------------------------------
struct TcScratch {
  float* x_blk;
  float* ple_blk;
  float* val_blk;
  __nv_bfloat16* attn_blk;
  void* q;
  int64_t total;
};

static int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

TcScratch plan_tc(const cg_trunk_dims& dims, int64_t batch, int steps, unsigned char* base) {
  const int64_t nt = batch * steps, ntiles = (nt + kTile - 1) / kTile, rows = ntiles * kTile;
  const int64_t d = dims.d_model, P = dims.per_layer_dim, L = dims.n_layers;
  const int64_t kvw = static_cast<int64_t>(dims.n_kv_heads) * head_dim(dims), nv = value_layer_count(dims);
  TcScratch s{};
  int64_t at = 0;
  auto take = [&](int64_t bytes) {
    unsigned char* here = base ? base + at : nullptr;
    at = align256(at + bytes);
    return here;
  };
  s.x_blk = reinterpret_cast<float*>(take(rows * d * 4));
  s.ple_blk = reinterpret_cast<float*>(take(L * rows * P * 4));
  s.val_blk = reinterpret_cast<float*>(take(nv * rows * kvw * 4));
  s.attn_blk = reinterpret_cast<__nv_bfloat16*>(take(rows * d * 2));
  s.q = take(nt * d * 4);
  s.total = at;
  return s;
}

int64_t tc_layers_scratch_bytes(const cg_trunk_dims& dims, int64_t batch, int steps) {
  return plan_tc(dims, batch, steps, nullptr).total;
}

int launch_dense(TcParams& p, cudaStream_t s) {
  int max_n = 0;
  for (int i = 0; i < p.n_ops; ++i) max_n = p.ops[i].n > max_n ? p.ops[i].n : max_n;
  p.stage_bytes = max_n * 32;
  const int abytes = kTile * p.d * 2;
  int stages = p.stage_bytes ? (kSmemBudget - 2 * abytes) / p.stage_bytes : 1;
  p.stages = stages > kMaxStages ? kMaxStages : stages;
  if (p.stages < 2) return set_error(CG_ERR_ARGUMENT, "tensor-core dense layer does not fit in shared memory");
  const int smem = 2 * abytes + p.stages * p.stage_bytes;
  static int configured_smem[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (configured_smem[device & 63] < smem) {
    cudaError_t err = cudaFuncSetAttribute(tc_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "tc_dense_kernel smem: %s", cudaGetErrorString(err));
    configured_smem[device & 63] = smem;
  }
  tc_dense_kernel<<<static_cast<unsigned>(p.ntiles), kTcThreads, smem, s>>>(p);
  return check_launch("tc_dense_kernel");
}

__global__ void readout_norm_kernel(const float* __restrict__ x_blk, int d, int steps, int64_t batch,
                                    const int64_t* __restrict__ offsets, const float* __restrict__ w,
                                    const float* __restrict__ b, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t bi = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (bi >= batch) return;
  const int64_t row = bi * steps + offsets[bi];
  const int64_t tile = row / kTile;
  const int t = static_cast<int>(row % kTile);
  auto at = [&](int k) {
    const float4 e = reinterpret_cast<const float4*>(x_blk)[(tile * (d / 4) + k / 4) * kTile + t];
    const int l = k & 3;
    return l == 0 ? e.x : l == 1 ? e.y : l == 2 ? e.z : e.w;
  };
  float sum = 0.f;
  for (int k = lane; k < d; k += 32) sum += at(k);
  const float mean = warp_sum(sum) / d;
  float var = 0.f;
  for (int k = lane; k < d; k += 32) {
    const float c = at(k) - mean;
    var += c * c;
  }
  const float rstd = rsqrtf(warp_sum(var) / d + 1e-5f);
  for (int k = lane; k < d; k += 32) out[bi * d + k] = (at(k) - mean) * rstd * w[k] + b[k];
}

int run_tc_forward(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int64_t batch, int steps,
                   const int64_t* positions, const int64_t* key_lengths, const int64_t* rows, int span, void* k_pool,
                   void* v_pool, int kv_dtype, int64_t capacity, int max_len, const float* lookup, int lookup_width,
                   const float* x_in, const float* ple_in, const float* val_in, unsigned char* scratch,
                   int64_t scratch_bytes, const int64_t* readout_offsets, float* hidden_out, cudaStream_t s) {
  TcScratch w = plan_tc(dims, batch, steps, scratch);
  if (scratch_bytes < w.total) return set_error(CG_ERR_WORKSPACE, "tensor-core scratch too small");
  const int d = dims.d_model, f = dims.d_ff, H = dims.n_heads, KVH = dims.n_kv_heads, D = head_dim(dims);
  const int qw = qkv_width(dims);
  const int64_t nt = batch * steps;
  const int64_t layer_elems = capacity * KVH * static_cast<int64_t>(max_len) * D;
  const int esize = dtype_size(kv_dtype);
  auto kv_layer = [&](void* pool, int layer) {
    return static_cast<void*>(static_cast<unsigned char*>(pool) + layer * layer_elems * esize);
  };

  TcParams p{};
  p.d = d;
  p.f = f;
  p.H = H;
  p.KVH = KVH;
  p.D = D;
  p.L = dims.n_layers;
  p.P = dims.per_layer_dim;
  p.nv = value_layer_count(dims);
  p.kvw = KVH * D;
  p.qw = qw;
  p.nt = nt;
  p.ntiles = (nt + kTile - 1) / kTile;
  p.T = steps;
  p.x_blk = w.x_blk;
  p.ple_blk = w.ple_blk;
  p.val_blk = w.val_blk;
  p.attn_blk = w.attn_blk;
  p.q = w.q;
  p.q_dtype = kv_dtype;
  p.kv_dtype = kv_dtype;
  p.max_len = max_len;
  p.positions = positions;
  p.rows = rows;
  p.ple_scale = [&] {
    if (!p.P || p.P == d) return 1.f;
    return static_cast<float>(1.0 / std::sqrt(static_cast<double>((d + p.P - 1) / p.P)));
  }();

  auto qkv_op = [&](int layer) {
    GemmOp op{};
    op.w = layer_pack(dims, blob, L, layer).qkv;
    op.n = qw;
    op.ksteps = d / 16;
    op.tmem_col = 0;
    op.wait_a = 1;
    op.signal = 1;
    return op;
  };
  auto set_qkv_target = [&](int layer) {
    p.qkv_layer = layer;
    p.value_index = value_index(dims, layer);
    p.k_layer = kv_layer(k_pool, layer);
    p.v_layer = kv_layer(v_pool, layer);
    p.ln_next_w = part(blob, L, CG_PART_LN_ATTN_W, layer);
    p.ln_next_b = part(blob, L, CG_PART_LN_ATTN_B, layer);
  };

  // First kernel: conditioning (or the given conditioned streams) + layer 0's QKV.
  int rc;
  p.n_ops = 0;
  if (lookup) {
    p.mode = kFirstLookup;
    p.lookup = lookup;
    p.lookup_width = lookup_width;
    p.rms_w = part(blob, L, CG_PART_INPUT_NORM, 0);
    const int ple_w = dims.n_layers * dims.per_layer_dim;
    for (int c0 = 0; c0 < ple_w; c0 += 256) {
      GemmOp op{};
      op.w = blob_ptr<__nv_bfloat16>(blob, L.bf16_ple_context) + static_cast<int64_t>(c0) * d;
      op.n = ple_w - c0 < 256 ? ple_w - c0 : 256;
      op.ksteps = d / 16;
      op.tmem_col = 0;
      op.wait_a = 1;
      op.signal = 1;
      p.ops[p.n_ops++] = op;
    }
  } else {
    p.mode = kFirstConditioned;
    p.x_in = x_in;
    p.ple_in = ple_in;
    p.val_in = val_in;
  }
  p.ops[p.n_ops++] = qkv_op(0);
  set_qkv_target(0);
  p.layer = 0;
  p.has_next = 1;
  if ((rc = launch_dense(p, s))) return rc;

  for (int layer = 0; layer < dims.n_layers; ++layer) {
    AttnParams a{};
    a.q = w.q;
    a.q_dtype = kv_dtype;
    a.q_st = D;
    a.q_sh = static_cast<int64_t>(steps) * D;
    a.q_sb = static_cast<int64_t>(H) * steps * D;
    a.k = kv_layer(k_pool, layer);
    a.v = kv_layer(v_pool, layer);
    a.kv_dtype = kv_dtype;
    a.kv_pos = D;
    a.kv_head = static_cast<int64_t>(max_len) * D;
    a.kv_row = static_cast<int64_t>(KVH) * max_len * D;
    a.rows = rows;
    a.lengths = key_lengths;
    a.batch = batch;
    a.heads = H;
    a.kv_heads = KVH;
    a.steps = steps;
    a.group = H / KVH;
    a.head_dim = D;
    a.span = span;
    a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
    a.out = w.attn_blk;
    a.out_dtype = CG_BF16;
    a.out_blocked = 1;
    a.blocked_width = d;
    if ((rc = run_attention(a, s))) return rc;

    LayerPack lp = layer_pack(dims, blob, L, layer);
    p.mode = kLayer;
    p.layer = layer;
    p.has_next = layer + 1 < dims.n_layers;
    p.ln_mlp_w = part(blob, L, CG_PART_LN_MLP_W, layer);
    p.ln_mlp_b = part(blob, L, CG_PART_LN_MLP_B, layer);
    p.up_b = part(blob, L, CG_PART_UP_B, layer);
    p.down_b = part(blob, L, CG_PART_DOWN_B, layer);
    p.n_ops = 0;
    GemmOp out{};
    out.w = lp.out;
    out.n = d;
    out.ksteps = d / 16;
    out.tmem_col = 0;
    out.wait_a = 1;
    out.signal = 1;
    p.ops[p.n_ops++] = out;
    const int chunks = f / d;
    for (int c = 0; c < chunks; ++c) {
      GemmOp up{};
      up.w = lp.up + static_cast<int64_t>(c) * d * d;
      up.n = d;
      up.ksteps = d / 16;
      up.tmem_col = 256;
      up.wait_a = c == 0;
      up.signal = 1;
      p.ops[p.n_ops++] = up;
      GemmOp down{};
      down.w = lp.down + static_cast<int64_t>(c) * d * d;
      down.n = d;
      down.ksteps = d / 16;
      down.tmem_col = 0;
      down.a_src = 1;
      down.accumulate_first = c > 0;
      down.wait_a = 1;
      down.signal = c == chunks - 1;
      p.ops[p.n_ops++] = down;
    }
    if (p.has_next) {
      p.ops[p.n_ops++] = qkv_op(layer + 1);
      set_qkv_target(layer + 1);
    }
    if (p.n_ops > kMaxOps) return set_error(CG_ERR_ARGUMENT, "too many GEMM steps in one dense layer");
    if ((rc = launch_dense(p, s))) return rc;
  }
  readout_norm_kernel<<<static_cast<unsigned>((batch + 7) / 8), 256, 0, s>>>(
      w.x_blk, d, steps, batch, readout_offsets, part(blob, L, CG_PART_FINAL_W, 0), part(blob, L, CG_PART_FINAL_B, 0),
      hidden_out);
  return check_launch("readout_norm_kernel");
}

int tc_condition_ple(const cg_trunk_dims&, const void*, const BlobLayout&, const float*, const float*, int64_t, int64_t,
                     float*, cudaStream_t) {
  return set_error(CG_ERR_ARGUMENT, "tensor-core conditioning runs inside the fused forward");
}

}  // namespace cg
