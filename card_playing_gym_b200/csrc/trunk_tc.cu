// Tensor-core (tcgen05) dense layers of the bf16 ragged decode step.
//
// Reference arithmetic: cardgym/nn/trunk.py — condition 285-312 (RMSNorm, PLE context
// projection), DecoderBlock._qkv 141-152 (LN, fused QKV, value embedding),
// _finish 154-157 (out projection + residual, LN, GELU MLP + residual), _add_ple
// 318-333, and the KV append of kv_cache.py:84-105 with trunk.py:419-423's clamp.
//
// One CTA owns a tile of 128 row-tokens and carries it across a layer boundary:
//   attention(l) output -> out_proj -> x += . -> LN -> up (128-column chunks) -> GELU ->
//   down (accumulated over the chunks) -> x += . + b -> x += PLE(l) -> LN -> QKV(l+1)
//   -> q for attention(l+1), K/V appended to the pool.
// The MLP is double-buffered: up chunks alternate between two TMEM column ranges and their
// GELU outputs between two shared-memory H buffers, so the tensor core runs up(c+1) and
// down(c-1) while the epilogue warps compute GELU(c).
// Roles: warps 0-11 are epilogue warps (three threads per row, each holding a third of
// the row's columns); warp 12's lane 0 streams weight K-slices into a ring of 32 KB
// shared-memory stages with bulk async copies; warp 13 allocates tensor memory and its
// lane 0 issues tcgen05.mma (M=128, bf16 x bf16 -> fp32 in TMEM). The GEMM weights are
// pre-packed (tc_pack) so consecutive K=16 slices of a GEMM step are contiguous and
// already in the canonical operand layout.
//
// Activations between kernels live in a tile-blocked layout so that thread-per-row
// access is coalesced: element (row r, column k) of an fp32 [rows, width] array sits
// at float4 index ((tile * width/4 + k/4) * 128 + r % 128), lane k % 4; the
// attention output (the out-projection operand) is bf16 in the operand layout itself:
// tile block = width/8 chunks of [128 rows x 8 columns].
#include <cmath>

#include "launch_timer.cuh"
#include "tcgen05.cuh"
#include "trunk.h"

namespace cg {

constexpr int kTile = 128;
constexpr int kTcThreads = 14 * 32;  // 12 epilogue warps + producer warp + MMA warp
constexpr int kMaxOps = 16;
constexpr int kMaxStages = 16;
constexpr int kStageTarget = 30 * 1024;  // bytes per ring stage (one bulk copy): a whole 128-column up half
constexpr int kSmemBudget = 222 * 1024;  // dynamic shared memory; the static barriers and reductions need the rest of 227 KB
constexpr int kUpCols = 128;             // up-projection chunk: columns of d_ff per GELU hand-off
constexpr int kAccCols = 256;            // TMEM: [0, 256) out/down/QKV accumulator, then two up buffers
// GEMM completion signals (tcgen05.commit targets).
enum Signal { kSigNone = 0, kSigAcc = 1, kSigUp0 = 2, kSigUp1 = 3, kSigHFree0 = 4, kSigHFree1 = 5 };

enum TcMode { kLayer = 0, kFirstBlocked = 1, kFirstConditioned = 2 };

struct GemmOp {
  const __nv_bfloat16* w;  // packed K-slices: ksteps x [n rows x 16 columns]
  int n;
  int ksteps;
  int ks_per_stage;  // consecutive K-slices carried by one ring stage (one bulk copy)
  int tmem_col;
  int a_src;  // 0: A buffer, 1: H buffer 0, 2: H buffer 1
  int accumulate_first;
  int wait_a;
  int signal;  // Signal
};

struct TcParams {
  int mode, layer, qkv_layer, has_next;
  GemmOp ops[kMaxOps];
  int n_ops, n_ple_ops, stages, stage_bytes, hbytes, n_up;
  int d, f, H, KVH, D, L, P, nv, kvw, qw;
  int64_t nt, ntiles;
  int T;
  float* x_blk;
  float* ple_blk;
  float* val_blk;
  const __nv_bfloat16* attn_blk;
  void* q;
  int q_dtype;
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
  // Last layer: the final LayerNorm at each row's readout token goes straight to hidden_out.
  const float* final_w;
  const float* final_b;
  const int64_t* readout_offsets;
  float* hidden_out;
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

// The residual row, stored with an L2 evict-last policy: the next layer's kernel reads it back after
// the attention kernel between them has streamed the KV pool (evict-first) through L2.
__device__ __forceinline__ void store16_keep(float* base, int64_t tile, int width, int col, int t, const float (&v)[16],
                                             uint64_t policy) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(blk(base, tile, width, col + 4 * q, t)),
                 "f"(v[4 * q]), "f"(v[4 * q + 1]), "f"(v[4 * q + 2]), "f"(v[4 * q + 3]), "l"(policy)
                 : "memory");
}

// Bring `bytes` (a multiple of 16, 16-byte aligned) of global memory into L2 ahead of their use.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 16 consecutive floats from a 16-byte aligned parameter vector (staged in shared memory).
__device__ __forceinline__ void load16_vec(const float* src, float (&v)[16]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = reinterpret_cast<const float4*>(src)[q];
    v[4 * q] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
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

// ---- GELU of the bf16 MLP ------------------------------------------------------------------------------
// GELU(x) = x Phi(x), with 0.5 erfc(z) (z = |x| / sqrt 2) from Abramowitz & Stegun 7.1.26:
// erfc(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z), |error| <= 1.5e-7.
// The GELU's absolute error stays below 5e-7, far inside the bf16 rounding of its output (the
// down-projection operand); Phi(x) = 1 - 0.5 erfc(z) for x >= 0 and 0.5 erfc(z) below, so the
// negative tail keeps its relative accuracy instead of cancelling.
// Computed on two values at once: the additions, multiplications and fused multiply-adds run as
// Blackwell's packed fp32x2 operations (each lane rounded exactly as the scalar operation), the
// reciprocal and the exponential per value (MUFU). Returns the pair packed as bf16 (x.x in the
// low half), the down projection's operand.
__device__ __forceinline__ uint32_t gelu_bf16_pair(float2 x) {
  const float2 z = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), make_float2(0.70710678118654752f, 0.70710678118654752f));
  const float2 den = __ffma2_rn(make_float2(0.3275911f, 0.3275911f), z, make_float2(1.f, 1.f));
  float2 t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.x) : "f"(den.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.y) : "f"(den.y));
  float2 q = __ffma2_rn(t, make_float2(0.5f * 1.061405429f, 0.5f * 1.061405429f),
                        make_float2(0.5f * -1.453152027f, 0.5f * -1.453152027f));
  q = __ffma2_rn(q, t, make_float2(0.5f * 1.421413741f, 0.5f * 1.421413741f));
  q = __ffma2_rn(q, t, make_float2(0.5f * -0.284496736f, 0.5f * -0.284496736f));
  q = __ffma2_rn(q, t, make_float2(0.5f * 0.254829592f, 0.5f * 0.254829592f));
  // (-z * z) * log2(e) = -((z * z) * log2(e)): negation is exact, so the rounding is the scalar form's
  const float2 arg = __fmul2_rn(__fmul2_rn(z, z), make_float2(-1.4426950408889634f, -1.4426950408889634f));
  float2 e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.x) : "f"(arg.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e.y) : "f"(arg.y));
  const float2 c = __fmul2_rn(__fmul2_rn(q, t), e);
  const float2 one_minus = __ffma2_rn(c, make_float2(-1.f, -1.f), make_float2(1.f, 1.f));  // rn(1 - c)
  const float2 phi = make_float2(x.x >= 0.f ? one_minus.x : c.x, x.y >= 0.f ? one_minus.y : c.y);
  const float2 g = __fmul2_rn(x, phi);
  __nv_bfloat162 pair = __floats2bfloat162_rn(g.x, g.y);
  return *reinterpret_cast<uint32_t*>(&pair);
}

// ---- epilogue geometry ---------------------------------------------------------------------------------
// 12 epilogue warps; thread e belongs to warp w = e / 32. Warp w may only touch TMEM lanes
// 32 * (w % 4) .. + 31, so row t = 32 * (w % 4) + lane, and the three warps with the same w % 4
// split the row's columns in thirds (part qd = w / 4), in 16-column chunks. With the producer and
// MMA warps the CTA has 14 warps, at most 4 per SM sub-partition, so a thread may use 128
// registers: enough to hold its third of the residual row (<= 5 chunks, d <= 240) across a layer.
constexpr int kParts = 3;
constexpr int kEpiWarps = 4 * kParts;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kMaxRowChunks = 6;  // 16-column chunks of a d <= 288 row held per thread (5 up to d = 240)
constexpr int kProducerWarp = kEpiWarps;
constexpr int kMmaWarp = kEpiWarps + 1;

struct EpiThread {
  int t;   // row in the tile == TMEM lane
  int qd;  // column part
  uint32_t lane_tmem;
};

// This part's chunk range of a row of `width` columns.
__device__ __forceinline__ void part_chunks(int width, int qd, int& lo, int& hi) {
  const int chunks = width / 16;
  const int per = (chunks + kParts - 1) / kParts;
  lo = qd * per;
  hi = min(chunks, lo + per);
  if (lo > hi) lo = hi;
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory"); }

// Sum of `value` over the kParts threads that share row t.
__device__ __forceinline__ float row_sum(float value, const EpiThread& e, float (*red)[kTile]) {
  red[e.qd][e.t] = value;
  epi_sync();
  float total = 0.f;
#pragma unroll
  for (int q = 0; q < kParts; ++q) total += red[q][e.t];
  return total;
}

// LayerNorm (eps 1e-5, biased variance, mean then centred variance) of the row held in
// registers (this thread's chunks lo..hi-1 of d), written as bf16 into the operand buffer,
// or, with to_row, as fp32 into out_row (a row-major d-wide row; skipped when null). Every
// epilogue thread takes part (the row statistics go through named barriers).
template <int kRC>
__device__ void layer_norm_regs(const float (&x)[kRC][16], int lo, int hi, int d, const EpiThread& e,
                                const float* w, const float* b, unsigned char* abuf, float (*red)[kTile],
                                bool to_row = false, float* out_row = nullptr) {
  float part = 0.f;
#pragma unroll
  for (int c = 0; c < kRC; ++c)
    if (lo + c < hi)
#pragma unroll
      for (int i = 0; i < 16; ++i) part += x[c][i];
  const float mean = row_sum(part, e, red) / d;
  float sq = 0.f;
#pragma unroll
  for (int c = 0; c < kRC; ++c)
    if (lo + c < hi)
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float z = x[c][i] - mean;
        sq += z * z;
      }
  const float rstd = rsqrtf(row_sum(sq, e, red + kParts) / d + 1e-5f);
#pragma unroll
  for (int c = 0; c < kRC; ++c) {
    if (lo + c >= hi) continue;
    const int col = (lo + c) * 16;
    float wv[16], bv[16];
    load16_vec(w + col, wv);
    load16_vec(b + col, bv);
    float y[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) y[i] = (x[c][i] - mean) * rstd * wv[i] + bv[i];
    if (!to_row) {
      store_operand16(abuf, col, e.t, y);
    } else if (out_row) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<float4*>(out_row + col)[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
    }
  }
}

// ---- the QKV epilogue: q out, K/V (+ value embedding) into the pool ------------------------------------
// Eight consecutive values (a 16-byte fp16/bf16 piece) to base[off..off+7], off % 8 == 0.
__device__ __forceinline__ void store8(void* base, int64_t off, int dtype, const float* v) {
  if (dtype == CG_F32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(base) + off);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    return;
  }
  uint4 packed;
  uint32_t* words = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dtype == CG_F16) {
      __half2 h2 = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      words[i] = *reinterpret_cast<uint32_t*>(&h2);
    } else {
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      words[i] = *reinterpret_cast<uint32_t*>(&h2);
    }
  }
  *reinterpret_cast<uint4*>(static_cast<uint16_t*>(base) + off) = packed;
}

// Columns [0, H*D) are q, then K and V (kvw = KVH*D each). With D % 8 == 0 every 8-column
// piece lies inside one head, so it is 8 contiguous elements of q's [B, H, T, D] layout or
// of one pool position: one 16-byte store. val_tile: this tile's value-embedding block in
// shared memory (blocked layout, [kvw/4][128] float4), or null to read it from val_blk.
__device__ void qkv_epilogue(const TcParams& p, const EpiThread& e, int64_t tile, const float4* val_tile) {
  const int t = e.t;
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
  // Row bases; a piece adds h * T * D + dd (q) or kvh * max_len * D + dd (K/V).
  const int64_t q_row = (b * p.H * p.T + tt) * p.D;
  const int64_t kv_row = (cache_row * p.KVH * p.max_len + pos) * p.D;
  const int q_head = p.T * p.D, kv_head = p.max_len * p.D;
  const float4* val_rows = val_tile ? val_tile + t
                                    : reinterpret_cast<const float4*>(p.val_blk) +
                                          (static_cast<int64_t>(p.value_index) * p.ntiles + tile) * (p.kvw / 4) * kTile + t;
  int lo, hi;
  part_chunks(p.qw, e.qd, lo, hi);
  for (int c = lo; c < hi; c += 2) {
    const bool two = c + 1 < hi;
    float v[32];
    tc::tmem_ld_pair(e.lane_tmem + c * 16, two, v);
    if (!valid) continue;
#pragma unroll
    for (int piece = 0; piece < 4; ++piece) {
      if (piece >= 2 && !two) break;
      const int col = c * 16 + piece * 8;
      float* w = v + piece * 8;
      if (col < hd) {
        const int h = col / p.D, dd = col - h * p.D;
        store8(p.q, q_row + (h * q_head + dd), p.q_dtype, w);
        continue;
      }
      const int cc = col - hd;
      const int which = cc >= p.kvw ? 1 : 0;
      const int rem = cc - which * p.kvw;
      const int kvh = rem / p.D, dd = rem - kvh * p.D;
      if (which && p.value_index >= 0) {
        const float4 e0 = val_rows[(rem / 4) * kTile];
        const float4 e1 = val_rows[(rem / 4 + 1) * kTile];
        w[0] += e0.x;
        w[1] += e0.y;
        w[2] += e0.z;
        w[3] += e0.w;
        w[4] += e1.x;
        w[5] += e1.y;
        w[6] += e1.z;
        w[7] += e1.w;
      }
      store8(which ? p.v_layer : p.k_layer, kv_row + (kvh * kv_head + dd), p.kv_dtype, w);
    }
  }
}

// ---- epilogue warps ----------------------------------------------------------------------------------------
template <int kRC>
__device__ void dense_epilogue(const TcParams& p, unsigned char* abuf, unsigned char* h0, unsigned char* h1, uint32_t tmem,
                               uint64_t* a_ready_bar, uint32_t publish_to, uint64_t* acc_ready_bar, uint64_t* up_ready_bar,
                               uint64_t* h_free_bar, uint64_t* attn_full_bar, uint64_t* val_full_bar, int abytes,
                               float (*red)[kTile], float* prm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tile = blockIdx.x;
  // The layer's vectors, staged once in shared memory (constant parameters: loaded while the
  // kernel before drains): [0,d) LN_mlp w (first kernel: input RMSNorm gain), [d,2d) LN_mlp b,
  // [2d,3d) down bias, [3d,5d) the next LN (last layer: the final LN), [5d,5d+f) up bias.
  {
    const int dd = p.d;
    for (int i = threadIdx.x; i < 5 * dd + p.f; i += kEpiThreads) {
      const int which = i < 5 * dd ? i / dd : 5;
      const float* src = which == 0   ? (p.mode == kLayer ? p.ln_mlp_w : p.rms_w)
                         : which == 1 ? p.ln_mlp_b
                         : which == 2 ? p.down_b
                         : which == 3 ? (p.has_next ? p.ln_next_w : p.final_w)
                         : which == 4 ? (p.has_next ? p.ln_next_b : p.final_b)
                                      : p.up_b;
      const int k = which < 5 ? i - which * dd : i - 5 * dd;
      prm[i] = src ? src[k] : 0.f;
    }
  }
  if (threadIdx.x == 0 && p.mode == kLayer) {
    // Written by the wave's first kernel, long complete: this layer's PLE tile and the next
    // QKV's value-embedding tile, read late in this kernel.
    if (p.P)
      prefetch_l2(blk(p.ple_blk, static_cast<int64_t>(p.layer) * p.ntiles + blockIdx.x, p.P, 0, 0),
                  static_cast<uint32_t>(kTile * p.P * 4));
    if (p.has_next && p.value_index >= 0)
      prefetch_l2(reinterpret_cast<const float4*>(p.val_blk) +
                      (static_cast<int64_t>(p.value_index) * p.ntiles + blockIdx.x) * (p.kvw / 4) * kTile,
                  static_cast<uint32_t>(kTile * p.kvw * 4));
  }
  pdl_wait();  // the epilogue reads and writes what earlier kernels of the stream touch
  pdl_trigger();
  EpiThread e;
  e.t = (warp & 3) * 32 + lane;
  e.qd = warp >> 2;  // 0 .. kParts-1
  e.lane_tmem = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
  const int t = e.t;
  const int64_t row = tile * kTile + t;
  const bool valid = row < p.nt;
  const int d = p.d;
  int lo, hi;  // this thread's 16-column chunks of a d-wide row
  part_chunks(d, e.qd, lo, hi);
  uint32_t acc_phase = 0;
  float x[kRC][16];
  float v16[16];
  // One thread waits on each mbarrier and arrives for the group; the others park on a
  // hardware named barrier instead of polling shared memory.
  auto publish = [&]() {  // operand written and TMEM reads done: hand over to the MMA warp
    tc::fence_async_smem();
    tc::fence_before_sync();
    epi_sync();
    if (threadIdx.x == 0) {
      if (publish_to)
        tc::bar_arrive_cluster(publish_to);  // the odd CTA of a pair publishes to the even CTA's issuer
      else
        tc::bar_arrive(a_ready_bar);
    }
  };
  auto group_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (threadIdx.x == 0) red[2 * kParts][0] = tc::bar_wait(bar, parity, code) ? 1.f : 0.f;
    epi_sync();
    return red[2 * kParts][0] != 0.f;
  };
  auto wait_acc = [&]() -> bool {
    if (!group_wait(acc_ready_bar, acc_phase, 0x403)) return false;
    acc_phase ^= 1u;
    tc::fence_after_sync();
    return true;
  };

  if (p.mode == kLayer) {
    // E0: the attention output tile is already in operand layout: one bulk copy.
    if (threadIdx.x == 0) {
      tc::bar_expect_tx(attn_full_bar, abytes);
      tc::bulk_g2s(abuf, reinterpret_cast<const unsigned char*>(p.attn_blk) + tile * abytes, abytes, attn_full_bar);
    }
    // The residual row goes into the accumulator columns of TMEM: the out-projection and
    // every down-projection accumulate onto it, so x += out and x += down need no epilogue
    // and the row never leaves TMEM inside the layer.
    // Every chunk's loads first, then the stores: a tensor-memory store is a compiler barrier, so
    // interleaving them would make the chunks' global loads one round trip each.
#pragma unroll
    for (int c = 0; c < kRC; ++c)
      if (lo + c < hi) load16(p.x_blk, tile, d, (lo + c) * 16, t, x[c]);
#pragma unroll
    for (int c = 0; c < kRC; ++c)
      if (lo + c < hi) tc::tmem_st16(e.lane_tmem + (lo + c) * 16, x[c]);
    tc::tmem_wait_st();
    if (!group_wait(attn_full_bar, 0, 0x404)) return;
    publish();
    // E1: LN_mlp(x + out_proj) -> A.
    if (!wait_acc()) return;
#pragma unroll
    for (int c = 0; c < kRC; ++c)
      if (lo + c < hi) tc::tmem_ld16(e.lane_tmem + (lo + c) * 16, x[c]);
    layer_norm_regs(x, lo, hi, d, e, prm, prm + d, abuf, red);
    publish();
    // E2: GELU of each up chunk into its H buffer. Chunk uc sits in TMEM buffer uc % 2; its
    // H buffer is free once down(uc - 2) has completed.
    uint32_t up_phase[2] = {0u, 0u}, free_phase[2] = {0u, 0u};
    for (int uc = 0; uc < p.n_up; ++uc) {
      const int buf = uc & 1;
      if (threadIdx.x == 0) {
        bool ok = tc::bar_wait(&up_ready_bar[buf], up_phase[buf], 0x406);
        if (ok && uc >= 2) ok = tc::bar_wait(&h_free_bar[buf], free_phase[buf], 0x407);
        red[2 * kParts][0] = ok ? 1.f : 0.f;
      }
      epi_sync();
      if (red[2 * kParts][0] == 0.f) return;
      up_phase[buf] ^= 1u;
      if (uc >= 2) free_phase[buf] ^= 1u;
      tc::fence_after_sync();
      const int width = min(kUpCols, p.f - uc * kUpCols);
      int plo, phi;
      part_chunks(width, e.qd, plo, phi);
      unsigned char* hb = buf ? h1 : h0;
      const float* bias_base = prm + 5 * d + uc * kUpCols;
      const uint32_t ucol = kAccCols + buf * kUpCols;
      for (int c = plo; c < phi; c += 2) {
        const bool two = c + 1 < phi;
        float bias[2][16];
        load16_vec(bias_base + c * 16, bias[0]);
        if (two) load16_vec(bias_base + c * 16 + 16, bias[1]);
        float v[32];
        tc::tmem_ld_pair(e.lane_tmem + ucol + c * 16, two, v);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && !two) break;
          uint32_t words[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            words[i] = gelu_bf16_pair(__fadd2_rn(make_float2(v[16 * h + 2 * i], v[16 * h + 2 * i + 1]),
                                                 make_float2(bias[h][2 * i], bias[h][2 * i + 1])));
          const int col = (c + h) * 16;
#pragma unroll
          for (int q = 0; q < 2; ++q)
            *reinterpret_cast<uint4*>(hb + (col / 8 + q) * (kTile * 16) + t * 16) =
                make_uint4(words[4 * q], words[4 * q + 1], words[4 * q + 2], words[4 * q + 3]);
        }
      }
      publish();
    }
    // E3: x (= x + out + down, in TMEM) + b + PLE(l); store; then LN_attn(l+1) -> A.
    // The bias and the PLE update do not depend on the GEMM: gather them while it runs.
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      if (lo + c >= hi) {
#pragma unroll
        for (int i = 0; i < 16; ++i) x[c][i] = 0.f;
        continue;
      }
      const int col = (lo + c) * 16;
      load16_vec(prm + 2 * d + col, x[c]);
      if (p.P) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const int k = (col + i) % p.P;  // P % 4 == 0: four columns share a float4
          const float4 ev = *blk(p.ple_blk, static_cast<int64_t>(p.layer) * p.ntiles + tile, p.P, k, t);
          x[c][i] = fmaf(ev.x, p.ple_scale, x[c][i]);
          x[c][i + 1] = fmaf(ev.y, p.ple_scale, x[c][i + 1]);
          x[c][i + 2] = fmaf(ev.z, p.ple_scale, x[c][i + 2]);
          x[c][i + 3] = fmaf(ev.w, p.ple_scale, x[c][i + 3]);
        }
      }
    }
    if (!wait_acc()) return;
    // Every GEMM that reads H has completed: H takes the next layer's value-embedding tile.
    const uint64_t keep_x = tc::make_policy_evict_last();
    const int vbytes = kTile * p.kvw * 4;
    const bool val_smem = p.has_next && p.value_index >= 0 && vbytes <= p.hbytes;
    if (val_smem && threadIdx.x == 0) {
      tc::bar_expect_tx(val_full_bar, vbytes);
      tc::bulk_g2s(h0, reinterpret_cast<const unsigned char*>(p.val_blk) +
                             (static_cast<int64_t>(p.value_index) * p.ntiles + tile) * vbytes,
                   vbytes, val_full_bar);
    }
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      if (lo + c >= hi) continue;
      const int col = (lo + c) * 16;
      tc::tmem_ld16(e.lane_tmem + col, v16);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[c][i] += v16[i];
      if (p.has_next) store16_keep(p.x_blk, tile, d, col, t, x[c], keep_x);
    }
    if (p.has_next) {
      layer_norm_regs(x, lo, hi, d, e, prm + 3 * d, prm + 4 * d, abuf, red);
      publish();
      if (val_smem && !group_wait(val_full_bar, 0, 0x405)) return;
      if (!wait_acc()) return;
      qkv_epilogue(p, e, tile, val_smem ? reinterpret_cast<const float4*>(h0) : nullptr);
    } else {
      // Final LayerNorm only at each row's readout token (trunk.py:426-429), straight to hidden.
      const int64_t b = row / p.T;
      const int tt = static_cast<int>(row - b * p.T);
      const bool readout = valid && (p.T == 1 || tt == p.readout_offsets[b]);
      layer_norm_regs(x, lo, hi, d, e, prm + 3 * d, prm + 4 * d, abuf, red, true, readout ? p.hidden_out + b * d : nullptr);
    }
    return;
  }

  // First kernel of a wave: conditioned x, PLE and value streams into blocked layout.
  const int ple_w = p.L * p.P;
  const int val_w = p.nv * p.kvw;
  const int64_t r = valid ? row : 0;
  if (p.mode == kFirstBlocked) {
    // The field-lookup kernel wrote the raw streams in blocked layout: x into x_blk, the PLE
    // lookup into ple_blk, the value lookup into val_blk (already final).
    // x = RMSNorm(lookup x) * gain (trunk.py:297-298, 104-115) -> x_blk and the A operand;
    // LN_attn(0)(x) -> H buffer 0, the QKV GEMM's operand.
#pragma unroll
    for (int c = 0; c < kRC; ++c)
      if (lo + c < hi) load16(p.x_blk, tile, d, (lo + c) * 16, t, x[c]);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < kRC; ++c)
      if (lo + c < hi)
#pragma unroll
        for (int i = 0; i < 16; ++i) ss += x[c][i] * x[c][i];
    const float inv = rsqrtf(row_sum(ss, e, red) / d + 1e-5f);
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      if (lo + c >= hi) continue;
      const int col = (lo + c) * 16;
      float gain[16];
      load16_vec(prm + col, gain);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[c][i] = x[c][i] * inv * gain[i];
      store16_keep(p.x_blk, tile, d, col, t, x[c], tc::make_policy_evict_last());
      store_operand16(abuf, col, t, x[c]);
    }
    layer_norm_regs(x, lo, hi, d, e, prm + 3 * d, prm + 4 * d, h0, red);
    // ple = (lookup + W_c x) / sqrt(2): each 256-column GEMM accumulates onto the raw PLE
    // lookup preloaded into its TMEM buffer (ops alternate between two buffers).
    const float inv_sqrt2 = 0.70710678118654752f;
    const int n_ple = p.n_ple_ops;
    auto ple_float4 = [&](int k) {  // the blocked float4 holding PLE column k (k % 4 == 0) of row t
      const int layer = k / p.P, kk = k - layer * p.P;
      return blk(p.ple_blk, static_cast<int64_t>(layer) * p.ntiles + tile, p.P, kk, t);
    };
    auto preload = [&](int o) {
      int plo, phi;
      part_chunks(p.ops[o].n, e.qd, plo, phi);
      for (int c = plo; c < phi; ++c) {
#pragma unroll
        for (int i = 0; i < 16; i += 4) {
          const float4 ev = *ple_float4(o * kAccCols + c * 16 + i);
          v16[i] = ev.x;
          v16[i + 1] = ev.y;
          v16[i + 2] = ev.z;
          v16[i + 3] = ev.w;
        }
        tc::tmem_st16(e.lane_tmem + (o & 1) * kAccCols + c * 16, v16);
      }
    };
    if (n_ple > 0) preload(0);
    if (n_ple > 1) preload(1);
    tc::tmem_wait_st();
    publish();
    uint32_t buf_phase[2] = {0u, 0u};
    for (int o = 0; o < n_ple; ++o) {
      const int buf = o & 1;
      if (!group_wait(&up_ready_bar[buf], buf_phase[buf], 0x406)) return;
      buf_phase[buf] ^= 1u;
      tc::fence_after_sync();
      int plo, phi;
      part_chunks(p.ops[o].n, e.qd, plo, phi);
      for (int c = plo; c < phi; ++c) {
        tc::tmem_ld16(e.lane_tmem + buf * kAccCols + c * 16, v16);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *ple_float4(o * kAccCols + c * 16 + i) = make_float4(v16[i] * inv_sqrt2, v16[i + 1] * inv_sqrt2,
                                                               v16[i + 2] * inv_sqrt2, v16[i + 3] * inv_sqrt2);
      }
      if (o + 2 < n_ple) {
        preload(o + 2);
        tc::tmem_wait_st();
        publish();
      }
    }
    if (n_ple > 0) publish();  // every PLE buffer is read: the QKV GEMM may overwrite them
    if (!wait_acc()) return;
    qkv_epilogue(p, e, tile, nullptr);  // the value streams came from the field lookup
    return;
  }
  {
#pragma unroll
    for (int c = 0; c < kRC; ++c) {
      if (lo + c >= hi) continue;
      const int col = (lo + c) * 16;
#pragma unroll
      for (int i = 0; i < 16; ++i) x[c][i] = p.x_in[r * d + col + i];
      store16_keep(p.x_blk, tile, d, col, t, x[c], tc::make_policy_evict_last());
    }
    for (int k = e.qd * 4; k < ple_w; k += 4 * kParts) {
      const float4 ev = *reinterpret_cast<const float4*>(p.ple_in + r * ple_w + k);
      *blk(p.ple_blk, static_cast<int64_t>(k / p.P) * p.ntiles + tile, p.P, k % p.P, t) = ev;
    }
    for (int k = e.qd * 4; k < val_w; k += 4 * kParts) {
      const float4 ev = *reinterpret_cast<const float4*>(p.val_in + r * val_w + k);
      *blk(p.val_blk, static_cast<int64_t>(k / p.kvw) * p.ntiles + tile, p.kvw, k % p.kvw, t) = ev;
    }
  }
  layer_norm_regs(x, lo, hi, d, e, prm + 3 * d, prm + 4 * d, abuf, red);
  publish();
  if (!wait_acc()) return;
  qkv_epilogue(p, e, tile, nullptr);  // the value streams were written by this CTA just above
}

// ---- the kernel ------------------------------------------------------------------------------------------
// kPairTiles: CTAs run in clusters of two on two SMs. Each CTA owns a 128-row tile; one M = 256
// tcgen05.mma issued by the even CTA covers both tiles, and each CTA's shared memory holds
// only half of every weight stage (B's N rows split in halves), so each SM streams half the
// weights. The odd CTA's MMA warp relays its stage arrivals to the even CTA; MMA completions
// are committed to the barriers of both CTAs; both epilogues publish to the even CTA.
constexpr bool kPairTiles = true;

// kRC: 16-column chunks of a row per epilogue thread (5 for d <= 240, 6 up to d = 288).
template <int kRC>
__global__ void __launch_bounds__(kTcThreads, 1) tc_dense_kernel(const __grid_constant__ TcParams p) {
  constexpr bool kPair = kPairTiles;
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], peer_full[kMaxStages];
  __shared__ __align__(8) uint64_t a_ready, acc_ready, attn_full, val_full, up_ready[2], h_free[2], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ float red[2 * kParts + 1][kTile];  // row reductions across a row's threads; last row: wait status

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? tc::cluster_ctarank() : 0u;
  const int abytes = kTile * p.d * 2;
  unsigned char* abuf = smem;
  unsigned char* h0 = smem + abytes;
  unsigned char* h1 = smem + abytes + p.hbytes;
  unsigned char* ring = smem + abytes + 2 * p.hbytes;
  float* prm = reinterpret_cast<float*>(ring + p.stages * p.stage_bytes);  // 5d + f floats

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      tc::bar_init(&full[s], 1);
      tc::bar_init(&empty[s], 1);
      tc::bar_init(&peer_full[s], 1);
    }
    tc::bar_init(&a_ready, kPair ? 2 : 1);  // both epilogues publish to the even CTA
    tc::bar_init(&acc_ready, 1);
    tc::bar_init(&attn_full, 1);
    tc::bar_init(&val_full, 1);
    tc::bar_init(&mma_done, 1);
    for (int b = 0; b < 2; ++b) {
      tc::bar_init(&up_ready[b], 1);
      tc::bar_init(&h_free[b], 1);
    }
    tc::bar_fence_init();
  }
  if (warp == kMmaWarp) {
    if (kPair) {
      tc::tmem_alloc_pair(&tmem_base, 512);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(&tmem_base, 512);
      tc::tmem_relinquish();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (kPair) tc::cluster_sync();  // barriers initialised and tensor memory allocated in both CTAs
  tc::fence_after_sync();
  const uint32_t tmem = tmem_base;
  auto commit = [&](uint64_t* bar) {
    if (kPair)
      tc::mma_commit_pair(bar);
    else
      tc::mma_commit(bar);
  };

  if (warp == kProducerWarp) {
    // ---- producer: weight K-slices into the ring, several slices per bulk copy ---------------------
    // A bulk copy has a fixed cost of ~0.2 us, so each stage carries up to 32 KB of consecutive
    // K-slices of one GEMM step (they are contiguous in the packed weights). In pair mode this
    // CTA loads its half of each slice (the packed op holds all its first-half slices, then
    // all its second-half slices).
    if (lane == 0) {
      const uint64_t keep = tc::make_policy_evict_last();
      const int stages = p.stages;
      int stage = 0;
      uint32_t lap = 0;  // completed passes over the ring
      for (int o = 0; o < p.n_ops; ++o) {
        const GemmOp& op = p.ops[o];
        const uint32_t slice = static_cast<uint32_t>(kPair ? op.n / 2 : op.n) * 32u;
        const unsigned char* src =
            reinterpret_cast<const unsigned char*>(op.w) + rank * slice * static_cast<uint32_t>(op.ksteps);
        for (int s = 0; s < op.ksteps; s += op.ks_per_stage) {
          const uint32_t bytes = slice * static_cast<uint32_t>(min(op.ks_per_stage, op.ksteps - s));
          // From the second pass on, the stage must have been released by its MMAs.
          if (lap > 0 && !tc::bar_wait(&empty[stage], (lap - 1) & 1u, 0x400)) goto producer_done;
          tc::bar_expect_tx(&full[stage], bytes);
          tc::bulk_g2s_hint(ring + stage * p.stage_bytes, src, bytes, &full[stage], keep);
          src += bytes;
          if (++stage == stages) {
            stage = 0;
            ++lap;
          }
        }
      }
    producer_done:;
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0 && rank == 1) {
      // ---- odd CTA of a pair: relay each stage's arrival to the even CTA's MMA issuer ------------------
      const int stages = p.stages;
      int stage = 0;
      uint32_t lap = 0;
      for (int o = 0; o < p.n_ops; ++o) {
        bool ok = true;
        for (int s0 = 0; s0 < p.ops[o].ksteps; s0 += p.ops[o].ks_per_stage) {
          if (!(ok = tc::bar_wait(&full[stage], lap & 1u, 0x408))) break;
          tc::bar_arrive_cluster(tc::map_shared(tc::smem_u32(&peer_full[stage]), 0));
          if (++stage == stages) {
            stage = 0;
            ++lap;
          }
        }
        if (!ok) break;
      }
      tc::bar_wait(&mma_done, 0, 0x409);  // the even CTA's MMAs into this CTA's TMEM have completed
    } else if (lane == 0) {
      // ---- MMA issuer ---------------------------------------------------------------------------------
      const int stages = p.stages;
      const uint32_t ring_addr = tc::smem_u32(ring);
      int stage = 0;
      uint32_t lap = 0;
      uint32_t a_phase = 0;
      for (int o = 0; o < p.n_ops; ++o) {
        const GemmOp op = p.ops[o];
        if (op.wait_a) {
          if (!(kPair ? tc::bar_wait_cluster(&a_ready, a_phase, 0x401) : tc::bar_wait(&a_ready, a_phase, 0x401)))
            break;
          a_phase ^= 1u;
          tc::fence_after_sync();
        }
        const uint32_t a_addr = tc::smem_u32(op.a_src == 0 ? abuf : (op.a_src == 1 ? h0 : h1));
        const uint32_t slice = static_cast<uint32_t>(kPair ? op.n / 2 : op.n) * 32u;
        const uint32_t idesc = tc::idesc_bf16(kPair ? 256 : 128, op.n <= 256 ? op.n : 256);
        const uint32_t idesc_rest = tc::idesc_bf16(128, op.n > 256 ? op.n - 256 : 16);
        bool ok = true;
        for (int s0 = 0; s0 < op.ksteps; s0 += op.ks_per_stage) {
          if (!(ok = tc::bar_wait(&full[stage], lap & 1u, 0x402))) break;
          if (kPair && !(ok = tc::bar_wait_cluster(&peer_full[stage], lap & 1u, 0x40a))) break;
          tc::fence_after_sync();
          const int end = min(op.ksteps, s0 + op.ks_per_stage);
          // One thread issues every MMA while the epilogue warps keep the SM's issue slots busy, so
          // the loop is kept to the MMA itself: both descriptors are built once per stage and
          // stepped by a K-slice (the 14-bit address field, in 16-byte units, never carries: shared
          // memory addresses stay below 2^18).
          uint64_t a_desc = tc::smem_desc(a_addr + 2 * s0 * (kTile * 16), kTile * 16, 128);
          uint64_t b_desc = tc::smem_desc(ring_addr + stage * p.stage_bytes, 128, 256);
          constexpr uint64_t a_step = (2 * kTile * 16) >> 4;
          const uint64_t b_step = slice >> 4;
          const uint32_t d_tmem = tmem + op.tmem_col;
          for (int s = s0; s < end; ++s) {
            const uint32_t acc = (s > 0 || op.accumulate_first) ? 1u : 0u;
            if (kPair) {
              tc::mma_bf16_pair(d_tmem, a_desc, b_desc, idesc, acc);
            } else {
              tc::mma_bf16(d_tmem, a_desc, b_desc, idesc, acc);
              if (op.n > 256) tc::mma_bf16(d_tmem + 256, a_desc, b_desc + ((32 * 256) >> 4), idesc_rest, acc);
            }
            a_desc += a_step;
            b_desc += b_step;
          }
          commit(&empty[stage]);
          if (++stage == stages) {
            stage = 0;
            ++lap;
          }
        }
        if (!ok) break;
        switch (op.signal) {
          case kSigAcc: commit(&acc_ready); break;
          case kSigUp0: commit(&up_ready[0]); break;
          case kSigUp1: commit(&up_ready[1]); break;
          case kSigHFree0: commit(&h_free[0]); break;
          case kSigHFree1: commit(&h_free[1]); break;
          default: break;
        }
      }
      // Every MMA issued (into both CTAs' TMEM in pair mode) completes before anyone deallocates.
      commit(&mma_done);
      tc::bar_wait(&mma_done, 0, 0x409);
    }
  } else {
    const uint32_t publish_to = kPair && rank == 1 ? tc::map_shared(tc::smem_u32(&a_ready), 0) : 0u;
    dense_epilogue<kRC>(p, abuf, h0, h1, tmem, &a_ready, publish_to, &acc_ready, up_ready, h_free, &attn_full, &val_full,
                   abytes, red, prm);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (kPair) tc::cluster_sync();  // neither CTA leaves while the other may still reach its memory
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    if (kPair)
      tc::tmem_dealloc_pair(tmem, 512);
    else
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
  const __nv_bfloat16* up;    // up chunk c (rows c*kUpCols.., K = d) at c * kUpCols * d
  const __nv_bfloat16* down;  // down chunk c (K = columns c*kUpCols..) at c * kUpCols * d
};

inline int up_chunks(const cg_trunk_dims& dims) { return (dims.d_ff + kUpCols - 1) / kUpCols; }
inline int up_width(const cg_trunk_dims& dims, int c) {
  return dims.d_ff - c * kUpCols < kUpCols ? dims.d_ff - c * kUpCols : kUpCols;
}

LayerPack layer_pack(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int layer) {
  const int64_t d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  const __nv_bfloat16* base = blob_ptr<__nv_bfloat16>(blob, L.bf16_layer_base + layer * L.bf16_layer_stride);
  return {base, base + q * d, base + q * d + d * d, base + q * d + d * d + f * d};
}

bool tc_layers_available(const cg_trunk_dims& dims) {
  const int d = dims.d_model, D = head_dim(dims), q = qkv_width(dims);
  if (d % 16 || d / 16 > kParts * kMaxRowChunks || dims.d_ff % 16 || q % 16 || q > 512 || D % 8) return false;
  if (d > kAccCols || 2 * up_chunks(dims) + 3 > kMaxOps) return false;
  if (q > 256 && (q - 256) % 16) return false;
  if (dims.per_layer_dim % 4 || (static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim) % 16) return false;
  if ((dims.n_kv_heads * D) % 4) return false;
  const int64_t abytes = static_cast<int64_t>(kTile) * d * 2;
  const int64_t hbytes = static_cast<int64_t>(kTile) * (dims.d_ff < kUpCols ? dims.d_ff : kUpCols) * 2;
  const int64_t stage = 32LL * (q > 256 ? q : 256);
  return abytes + 2 * hbytes + 2 * stage + (5LL * d + dims.d_ff) * 4 <= kSmemBudget;
}

int tc_pack(const cg_trunk_dims& dims, void* blob, const BlobLayout& L, cudaStream_t s) {
  const int d = dims.d_model, f = dims.d_ff, q = qkv_width(dims);
  // One GEMM step's weights [N x K]: in pair mode as two [N/2 x K] halves one after the other
  // (the even CTA of a pair loads the first half's slices, the odd CTA the second's).
  auto pack = [&](const float* w, int ldw, int n0, int N, int k0, int K, __nv_bfloat16* dst) -> int {
    const int parts = kPairTiles ? 2 : 1;
    const int rows = N / parts;
    for (int h = 0; h < parts; ++h) {
      const int64_t total = static_cast<int64_t>(rows) * K;
      const unsigned blocks = static_cast<unsigned>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
      pack_kernel<<<blocks, 256, 0, s>>>(w, ldw, n0 + h * rows, rows, k0, K, dst + h * total);
      const int rc = check_launch("pack_kernel");
      if (rc) return rc;
    }
    return static_cast<int>(CG_OK);
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
    // QKV as two GEMM steps of <= 256 output columns: rows [0, 256) then [256, q).
    const int qa = q < 256 ? q : 256;
    if ((rc = pack(part(blob, L, CG_PART_QKV, layer), d, 0, qa, 0, d, const_cast<__nv_bfloat16*>(lp.qkv)))) return rc;
    if (q > 256 && (rc = pack(part(blob, L, CG_PART_QKV, layer), d, 256, q - 256, 0, d,
                             const_cast<__nv_bfloat16*>(lp.qkv) + static_cast<int64_t>(256) * d)))
      return rc;
    if ((rc = pack(part(blob, L, CG_PART_OUT, layer), d, 0, d, 0, d, const_cast<__nv_bfloat16*>(lp.out)))) return rc;
    for (int c = 0; c < up_chunks(dims); ++c) {
      const int w = up_width(dims, c);
      if ((rc = pack(part(blob, L, CG_PART_UP, layer), d, c * kUpCols, w, 0, d,
                     const_cast<__nv_bfloat16*>(lp.up) + static_cast<int64_t>(c) * kUpCols * d)))
        return rc;
      if ((rc = pack(part(blob, L, CG_PART_DOWN, layer), f, 0, d, c * kUpCols, w,
                     const_cast<__nv_bfloat16*>(lp.down) + static_cast<int64_t>(c) * kUpCols * d)))
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

// Tiles of 128 row-tokens; an even number in pair mode (a pair's odd CTA may hold no rows).
static int64_t padded_tiles(int64_t nt) {
  const int64_t tiles = (nt + kTile - 1) / kTile;
  return kPairTiles ? (tiles + 1) / 2 * 2 : tiles;
}

TcScratch plan_tc(const cg_trunk_dims& dims, int64_t batch, int steps, unsigned char* base) {
  const int64_t nt = batch * steps, ntiles = padded_tiles(nt), rows = ntiles * kTile;
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

// Where the field lookup writes its blocked raw streams for the first dense kernel.
void tc_input_streams(const cg_trunk_dims& dims, int64_t batch, int steps, unsigned char* scratch, float** x_blk,
                      float** ple_blk, float** val_blk, int64_t* ntiles) {
  const TcScratch w = plan_tc(dims, batch, steps, scratch);
  *x_blk = w.x_blk;
  *ple_blk = w.ple_blk;
  *val_blk = w.val_blk;
  *ntiles = padded_tiles(batch * steps);
}

int64_t tc_layers_scratch_bytes(const cg_trunk_dims& dims, int64_t batch, int steps) {
  return plan_tc(dims, batch, steps, nullptr).total;
}

namespace {
LaunchTimer g_dense_timer;
}  // namespace

int launch_dense_kernel(TcParams& p, cudaStream_t s);

int launch_dense(TcParams& p, cudaStream_t s) {
  const bool recorded = g_dense_timer.begin(s);
  const int rc = launch_dense_kernel(p, s);
  g_dense_timer.end(s, recorded);
  return rc;
}

int launch_dense_kernel(TcParams& p, cudaStream_t s) {
  // Ring stages of up to 32 KB (several consecutive K-slices each); as many as fit.
  const int abytes = kTile * p.d * 2;
  const int split = kPairTiles ? 2 : 1;  // a pair's CTA holds half of each K-slice
  int max_slice = 0;
  for (int i = 0; i < p.n_ops; ++i) max_slice = p.ops[i].n / split * 32 > max_slice ? p.ops[i].n / split * 32 : max_slice;
  p.stage_bytes = max_slice > kStageTarget ? max_slice : kStageTarget;
  const int fixed = abytes + 2 * p.hbytes + (5 * p.d + p.f) * 4;  // operands + staged layer vectors
  int stages = (kSmemBudget - fixed) / p.stage_bytes;
  if (stages < 2) {
    p.stage_bytes = max_slice;
    stages = (kSmemBudget - fixed) / p.stage_bytes;
  }
  p.stages = stages > kMaxStages ? kMaxStages : stages;
  if (p.stages < 2) return set_error(CG_ERR_ARGUMENT, "tensor-core dense layer does not fit in shared memory");
  for (int i = 0; i < p.n_ops; ++i) {
    const int per = p.stage_bytes / (p.ops[i].n / split * 32);
    p.ops[i].ks_per_stage = per < p.ops[i].ksteps ? per : p.ops[i].ksteps;
  }
  const int smem = fixed + p.stages * p.stage_bytes;
  if ((abytes + 2 * p.hbytes + p.stages * p.stage_bytes) % 16)
    return set_error(CG_ERR_ARGUMENT, "tensor-core dense layer: unaligned shared-memory layout");
  const bool wide = p.d / 16 > kParts * 5;  // rows of more than 15 chunks: six per thread
  auto kernel = wide ? tc_dense_kernel<6> : tc_dense_kernel<5>;
  static int configured_smem[2][64] = {{0}};
  int device = 0;
  cudaGetDevice(&device);
  if (configured_smem[wide][device & 63] < smem) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "tc_dense_kernel smem: %s", cudaGetErrorString(err));
    configured_smem[wide][device & 63] = smem;
  }
  // The producer warp streams only the constant packed weights, so it starts at once; the
  // epilogue warps wait for the kernel before (pdl_wait in dense_epilogue).
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(p.ntiles));
  config.blockDim = dim3(kTcThreads);
  config.dynamicSmemBytes = smem;
  config.stream = s;
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attribute[0].val.programmaticStreamSerializationAllowed = 1;
  attribute[1].id = cudaLaunchAttributeClusterDimension;
  attribute[1].val.clusterDim.x = kPairTiles ? 2 : 1;
  attribute[1].val.clusterDim.y = 1;
  attribute[1].val.clusterDim.z = 1;
  config.attrs = attribute;
  config.numAttrs = 2;
  cudaError_t err = cudaLaunchKernelEx(&config, kernel, p);
  if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "tc_dense_kernel launch: %s", cudaGetErrorString(err));
  return check_launch("tc_dense_kernel");
}

int run_tc_forward(const cg_trunk_dims& dims, const void* blob, const BlobLayout& L, int64_t batch, int steps,
                   const int64_t* positions, const int64_t* key_lengths, const int64_t* rows, int span, void* k_pool,
                   void* v_pool, int kv_dtype, int64_t capacity, int max_len, bool lookup_blocked,
                   const float* x_in, const float* ple_in, const float* val_in, unsigned char* scratch,
                   int64_t scratch_bytes, const int64_t* readout_offsets, float* hidden_out, int* attn_counters,
                   cudaStream_t s) {
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
  p.ntiles = padded_tiles(nt);
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
  p.final_w = part(blob, L, CG_PART_FINAL_W, 0);
  p.final_b = part(blob, L, CG_PART_FINAL_B, 0);
  p.readout_offsets = readout_offsets;
  p.hidden_out = hidden_out;
  p.hbytes = kTile * (f < kUpCols ? f : kUpCols) * 2;
  p.n_up = up_chunks(dims);
  p.ple_scale = [&] {
    if (!p.P || p.P == d) return 1.f;
    return static_cast<float>(1.0 / std::sqrt(static_cast<double>((d + p.P - 1) / p.P)));
  }();

  auto push_qkv = [&](int layer) {
    const __nv_bfloat16* w = layer_pack(dims, blob, L, layer).qkv;
    GemmOp op{};
    op.w = w;
    op.n = qw < 256 ? qw : 256;
    op.ksteps = d / 16;
    op.tmem_col = 0;
    op.wait_a = 1;
    op.signal = qw <= 256 ? kSigAcc : kSigNone;
    p.ops[p.n_ops++] = op;
    if (qw > 256) {
      GemmOp rest{};
      rest.w = w + static_cast<int64_t>(256) * d;
      rest.n = qw - 256;
      rest.ksteps = d / 16;
      rest.tmem_col = 256;
      rest.signal = kSigAcc;
      p.ops[p.n_ops++] = rest;
    }
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
  if (lookup_blocked) {
    // The field lookup wrote the raw streams into this scratch in blocked layout; the PLE
    // context GEMMs (256 columns each) accumulate onto the raw PLE lookup the epilogue
    // preloads into alternating TMEM buffers.
    p.mode = kFirstBlocked;
    p.rms_w = part(blob, L, CG_PART_INPUT_NORM, 0);
    const int ple_w = dims.n_layers * dims.per_layer_dim;
    for (int c0 = 0, o = 0; c0 < ple_w; c0 += kAccCols, ++o) {
      GemmOp op{};
      op.w = blob_ptr<__nv_bfloat16>(blob, L.bf16_ple_context) + static_cast<int64_t>(c0) * d;
      op.n = ple_w - c0 < kAccCols ? ple_w - c0 : kAccCols;
      op.ksteps = d / 16;
      op.tmem_col = (o & 1) * kAccCols;
      op.accumulate_first = 1;
      op.wait_a = o != 1;  // op 0: the operands; op o >= 2: buffer o % 2 consumed and reloaded
      op.signal = (o & 1) ? kSigUp1 : kSigUp0;
      p.ops[p.n_ops++] = op;
    }
  } else {
    p.mode = kFirstConditioned;
    p.x_in = x_in;
    p.ple_in = ple_in;
    p.val_in = val_in;
  }
  p.n_ple_ops = p.n_ops;
  push_qkv(0);
  if (lookup_blocked)
    for (int o = p.n_ple_ops; o < p.n_ops; ++o) p.ops[o].a_src = 1;  // LN_attn(0)(x) sits in H buffer 0
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
    a.counter = attn_counters + layer;
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
    p.n_ple_ops = 0;
    GemmOp out{};
    out.w = lp.out;
    out.n = d;
    out.ksteps = d / 16;
    out.tmem_col = 0;
    out.accumulate_first = 1;  // onto the residual row the epilogue put in these columns
    out.wait_a = 1;
    out.signal = kSigAcc;
    p.ops[p.n_ops++] = out;
    // MLP, double-buffered: up(0), up(1), then per chunk c: down(c) (after GELU(c)), up(c+2).
    const int n_up = p.n_up;
    auto push_up = [&](int c) {
      GemmOp up{};
      up.w = lp.up + static_cast<int64_t>(c) * kUpCols * d;
      up.n = up_width(dims, c);
      up.ksteps = d / 16;
      up.tmem_col = kAccCols + (c & 1) * kUpCols;
      up.wait_a = c == 0;  // LN_mlp(x) in the A buffer
      up.signal = (c & 1) ? kSigUp1 : kSigUp0;
      p.ops[p.n_ops++] = up;
    };
    push_up(0);
    if (n_up > 1) push_up(1);
    for (int c = 0; c < n_up; ++c) {
      GemmOp down{};
      down.w = lp.down + static_cast<int64_t>(c) * kUpCols * d;
      down.n = d;
      down.ksteps = up_width(dims, c) / 16;
      down.tmem_col = 0;
      down.a_src = 1 + (c & 1);
      down.accumulate_first = 1;  // onto x + out
      down.wait_a = 1;  // GELU(c) in H buffer c % 2
      down.signal = c == n_up - 1 ? kSigAcc : (c + 2 < n_up ? ((c & 1) ? kSigHFree1 : kSigHFree0) : kSigNone);
      p.ops[p.n_ops++] = down;
      if (c + 2 < n_up) push_up(c + 2);
    }
    if (p.has_next) {
      push_qkv(layer + 1);
      set_qkv_target(layer + 1);
    }
    if (p.n_ops > kMaxOps) return set_error(CG_ERR_ARGUMENT, "too many GEMM steps in one dense layer");
    if ((rc = launch_dense(p, s))) return rc;
  }
  return CG_OK;  // the last layer's epilogue wrote the readout hidden states
}

int tc_condition_ple(const cg_trunk_dims&, const void*, const BlobLayout&, const float*, const float*, int64_t, int64_t,
                     float*, cudaStream_t) {
  return set_error(CG_ERR_ARGUMENT, "tensor-core conditioning runs inside the fused forward");
}

}  // namespace cg

extern "C" int cg_dense_profiling(int enable, int capacity) {
  return cg::g_dense_timer.configure(enable, capacity, "cg_dense_profiling");
}

extern "C" int cg_dense_timings(float* ms_out, int max_count) { return cg::g_dense_timer.timings(ms_out, max_count); }
