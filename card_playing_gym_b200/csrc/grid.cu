// The piquet card grid: per-card features of a token's 32 card codes.
//
// Reference: cardgym/games/piquet/model.py:180-240 (`CardGrid.cards`), 129-177 (`GridBlock`),
// 118-126 (`GridNorm`). For one token, the 4 x 8 grid of cards (card = suit * 8 + rank) starts
// as code_emb[code] + rank_emb[rank] (fp32) and goes through `blocks` residual blocks:
//   rows   = RMSNorm(grid)                                        per card, over the width
//   along  = conv over ranks (3 taps, zero-padded) of rows, + bias  32 cards x 64 hidden
//   across = (mean over suits of rows) @ W_across                   8 ranks x 64 hidden
//   grid  += out(GELU(along + across[rank])) + bias                 32 cards x 32 width
// then a final RMSNorm. The reference runs this under bf16 autocast in its rollouts: every
// Linear / matmul output (with its bias) is rounded to bf16, as are their sum and the GELU,
// while the residual grid and the norms stay fp32. This kernel computes exactly that form:
// bf16 tensor-core operands (mma.sync m16n8k16), fp32 accumulation, the same rounding points.
//
// One warp per token: the grid lives in registers in the MMA accumulator layout (two m16
// tiles of cards x four n8 tiles of width); the normalised rows go through shared memory once
// (zero-padded ranks, so the convolution is three 32-wide k-blocks of an m16n8k16 GEMM read
// by ldmatrix); the GELU output feeds the output GEMM straight from registers. Weights sit in
// shared memory in bf16, [n][k] rows padded so ldmatrix rows hit distinct banks.
#include "common.cuh"

namespace cg {
namespace {

constexpr int kGridWarps = 8;
constexpr int kGW = 32;        // card width
constexpr int kGH = 64;        // block hidden width
constexpr int kGSuits = 4, kGRanks = 8, kGCards = 32;
constexpr int kGMaxBlocks = 4;
constexpr int kGMaxCodes = 16;
constexpr int kConvK = 3 * kGW;       // 96: three rank taps x width
constexpr int kConvStride = kConvK + 8;  // bf16 per conv weight row (208 bytes)
constexpr int kAcrossStride = kGW + 8;   // 80 bytes
constexpr int kOutStride = kGH + 8;      // 144 bytes
constexpr int kRowStride = kGW + 8;      // normed / pooled rows (80 bytes)

struct GridBlockSmem {
  __nv_bfloat16 conv[kGH * kConvStride];     // [hidden n][tap * 32 + width k]
  __nv_bfloat16 across[kGH * kAcrossStride];  // [hidden n][width k]
  __nv_bfloat16 out[kGW * kOutStride];       // [width n][hidden k]
  float norm[kGW];
  float conv_b[kGH];  // bf16-rounded (autocast casts the bias with the weight)
  float out_b[kGW];
};

struct GridWarpSmem {
  __nv_bfloat16 normed[kGSuits * (kGRanks + 2) * kRowStride];  // ranks -1..8, the outer two zero
  __nv_bfloat16 pooled[16 * kRowStride];                       // 8 ranks, rows 8..15 zero
};

struct GridSmem {
  float code[kGMaxCodes * kGW];
  float rank[kGRanks * kGW];
  float final_norm[kGW];
  GridBlockSmem block[kGMaxBlocks];
  GridWarpSmem warp[kGridWarps];
};

__device__ __forceinline__ uint32_t gsmem(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void g_ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void g_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ int64_t grid_code(const void* codes, int dtype, int64_t i) {
  if (dtype == CG_I16) return static_cast<const int16_t*>(codes)[i];
  if (dtype == CG_I32) return static_cast<const int32_t*>(codes)[i];
  return static_cast<const int64_t*>(codes)[i];
}

// RMSNorm of the rows this lane holds (rows gid and gid + 8 of both m16 tiles), in place into
// `out` (fp32): the row's 32 values are spread over the four lanes of a quad.
__device__ __forceinline__ void grid_rms(const float (&g)[2][4][4], const float* weight, int tid4,
                                         float (&out)[2][4][4]) {
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) ss += g[mt][j][2 * hf] * g[mt][j][2 * hf] + g[mt][j][2 * hf + 1] * g[mt][j][2 * hf + 1];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float rs = rsqrtf(ss * (1.f / kGW) + 1e-5f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = 8 * j + 2 * tid4;
        out[mt][j][2 * hf] = g[mt][j][2 * hf] * rs * weight[col];
        out[mt][j][2 * hf + 1] = g[mt][j][2 * hf + 1] * rs * weight[col + 1];
      }
    }
  }
}

__global__ void __launch_bounds__(kGridWarps * 32) card_grid_kernel(const cg_card_grid_weights w, const void* codes,
                                                                     int codes_dtype, int64_t n, int64_t stride,
                                                                     float* cards) {
  extern __shared__ __align__(16) unsigned char grid_smem_raw[];
  GridSmem& S = *reinterpret_cast<GridSmem*>(grid_smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tid4 = lane & 3;
  const int nblocks = w.blocks;

  // Stage the weights (bf16 GEMM operands in [n][k] rows; fp32 norms, bf16-rounded biases).
  for (int i = tid; i < w.codes * kGW; i += blockDim.x) S.code[i] = w.code_emb[i];
  for (int i = tid; i < kGRanks * kGW; i += blockDim.x) S.rank[i] = w.rank_emb[i];
  for (int i = tid; i < kGW; i += blockDim.x) S.final_norm[i] = w.final_norm[i];
  for (int b = 0; b < nblocks; ++b) {
    GridBlockSmem& B = S.block[b];
    for (int i = tid; i < kGH * kGW * 3; i += blockDim.x) {  // conv weight [hidden][width][tap]
      const int hh = i / (kGW * 3), rem = i - hh * kGW * 3, wi = rem / 3, tap = rem - wi * 3;
      B.conv[hh * kConvStride + tap * kGW + wi] = __float2bfloat16_rn(w.conv_w[b][i]);
    }
    for (int i = tid; i < kGH * kGW; i += blockDim.x) {
      const int hh = i / kGW, wi = i - hh * kGW;
      B.across[hh * kAcrossStride + wi] = __float2bfloat16_rn(w.across_w[b][i]);
    }
    for (int i = tid; i < kGW * kGH; i += blockDim.x) {
      const int o = i / kGH, hh = i - o * kGH;
      B.out[o * kOutStride + hh] = __float2bfloat16_rn(w.out_w[b][i]);
    }
    for (int i = tid; i < kGW; i += blockDim.x) {
      B.norm[i] = w.norm_w[b][i];
      B.out_b[i] = bf16r(w.out_b[b][i]);
    }
    for (int i = tid; i < kGH; i += blockDim.x) B.conv_b[i] = bf16r(w.conv_b[b][i]);
  }
  // Zero the per-warp padding: ranks -1 and 8 of the normed rows, pooled rows 8..15.
  GridWarpSmem& Wp = S.warp[warp];
  for (int i = lane; i < kGSuits * (kGRanks + 2) * kRowStride; i += 32) Wp.normed[i] = __float2bfloat16_rn(0.f);
  for (int i = lane; i < 16 * kRowStride; i += 32) Wp.pooled[i] = __float2bfloat16_rn(0.f);
  pdl_wait();
  pdl_trigger();
  __syncthreads();

  for (int64_t token = static_cast<int64_t>(blockIdx.x) * kGridWarps + warp; token < n;
       token += static_cast<int64_t>(gridDim.x) * kGridWarps) {
    // Card codes: lane c holds card c's.
    int64_t code = grid_code(codes, codes_dtype, token * stride + lane);
    if (code < 0 || code >= w.codes) {
      raise_fault(0x230);
      code = 0;
    }
    const int my_code = static_cast<int>(code);
    // The grid in accumulator layout: g[mt][j][e] is card mt*16 + gid (+8 for e >= 2),
    // width column 8j + 2*tid4 (+1 for odd e).
    float g[2][4][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int card = mt * 16 + gid + 8 * hf;
        const int c = __shfl_sync(0xffffffffu, my_code, card);
        const float* ce = S.code + c * kGW;
        const float* re = S.rank + (card & 7) * kGW;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = 8 * j + 2 * tid4;
          g[mt][j][2 * hf] = ce[col] + re[col];
          g[mt][j][2 * hf + 1] = ce[col + 1] + re[col + 1];
        }
      }

    for (int b = 0; b < nblocks; ++b) {
      const GridBlockSmem& B = S.block[b];
      float nm[2][4][4];
      grid_rms(g, B.norm, tid4, nm);
      __syncwarp();  // the previous token's / block's reads of `normed` are done
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int card = mt * 16 + gid + 8 * hf, s = card >> 3, r = card & 7;
          __nv_bfloat16* row = Wp.normed + (s * (kGRanks + 2) + r + 1) * kRowStride;
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint32_t*>(row + 8 * j + 2 * tid4) = pack_bf16(nm[mt][j][2 * hf], nm[mt][j][2 * hf + 1]);
        }
      __syncwarp();
      // Suit means (the reference's [1, 4] matmul of 1/4: products exact, sums in fp32, one rounding).
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int idx = lane + 32 * q, r = idx >> 4, cp = idx & 15;
        float a = 0.f, c = 0.f;
#pragma unroll
        for (int s = 0; s < kGSuits; ++s) {
          const __nv_bfloat162 v =
              *reinterpret_cast<const __nv_bfloat162*>(Wp.normed + (s * (kGRanks + 2) + r + 1) * kRowStride + 2 * cp);
          const float2 f = __bfloat1622float2(v);
          a = fmaf(0.25f, f.x, a);
          c = fmaf(0.25f, f.y, c);
        }
        *reinterpret_cast<uint32_t*>(Wp.pooled + r * kRowStride + 2 * cp) = pack_bf16(a, c);
      }
      // Rank convolution: 32 cards x 64 hidden, k = tap * 32 + width.
      float acc[2][8][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;
#pragma unroll
      for (int tap = 0; tap < 3; ++tap) {
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          uint32_t a[2][4];
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int card = mt * 16 + (lane & 15), s = card >> 3, r = card & 7;
            g_ldmatrix_x4(a[mt][0], a[mt][1], a[mt][2], a[mt][3],
                          gsmem(Wp.normed + (s * (kGRanks + 2) + r + tap) * kRowStride + kh * 16 + (lane >> 4) * 8));
          }
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b0, b1, b2, b3;
            g_ldmatrix_x4(b0, b1, b2, b3,
                          gsmem(B.conv + (16 * np + (lane & 15)) * kConvStride + tap * kGW + kh * 16 + (lane >> 4) * 8));
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
              g_mma(acc[mt][2 * np], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b2);
              g_mma(acc[mt][2 * np + 1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b1, b3);
            }
          }
        }
      }
      __syncwarp();  // every lane wrote its pooled values
      // Across-suit projection of the suit means: 8 ranks (rows gid) x 64 hidden.
      float xs[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) xs[nt][0] = xs[nt][1] = xs[nt][2] = xs[nt][3] = 0.f;
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) {
        uint32_t a0, a1, a2, a3;
        g_ldmatrix_x4(a0, a1, a2, a3, gsmem(Wp.pooled + (lane & 15) * kRowStride + kh * 16 + (lane >> 4) * 8));
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          g_ldmatrix_x4(b0, b1, b2, b3,
                        gsmem(B.across + (16 * np + (lane & 15)) * kAcrossStride + kh * 16 + (lane >> 4) * 8));
          g_mma(xs[2 * np], a0, a1, a2, a3, b0, b2);
          g_mma(xs[2 * np + 1], a0, a1, a2, a3, b1, b3);
        }
      }
      // mixed = bf16(bf16(along + bias) + bf16(across[rank])); GELU rounded to bf16. Rows gid
      // and gid + 8 of both m16 tiles are rank gid, whose across row this lane holds.
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = 8 * nt + 2 * tid4;
        const float x0 = bf16r(xs[nt][0]), x1 = bf16r(xs[nt][1]);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          acc[mt][nt][0] = bf16r(bf16r(acc[mt][nt][0] + B.conv_b[col]) + x0);
          acc[mt][nt][1] = bf16r(bf16r(acc[mt][nt][1] + B.conv_b[col + 1]) + x1);
          acc[mt][nt][2] = bf16r(bf16r(acc[mt][nt][2] + B.conv_b[col]) + x0);
          acc[mt][nt][3] = bf16r(bf16r(acc[mt][nt][3] + B.conv_b[col + 1]) + x1);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = acc[mt][nt][e];
            acc[mt][nt][e] = 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
          }
        }
      }
      // Output layer from registers (the accumulator pairs are the A fragments), + bias, rounded.
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        float o[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t a0 = pack_bf16(acc[mt][2 * j][0], acc[mt][2 * j][1]);
          const uint32_t a1 = pack_bf16(acc[mt][2 * j][2], acc[mt][2 * j][3]);
          const uint32_t a2 = pack_bf16(acc[mt][2 * j + 1][0], acc[mt][2 * j + 1][1]);
          const uint32_t a3 = pack_bf16(acc[mt][2 * j + 1][2], acc[mt][2 * j + 1][3]);
#pragma unroll
          for (int np = 0; np < 2; ++np) {
            uint32_t b0, b1, b2, b3;
            g_ldmatrix_x4(b0, b1, b2, b3,
                          gsmem(B.out + (16 * np + (lane & 15)) * kOutStride + 16 * j + (lane >> 4) * 8));
            g_mma(o[2 * np], a0, a1, a2, a3, b0, b2);
            g_mma(o[2 * np + 1], a0, a1, a2, a3, b1, b3);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const int col = 8 * nt + 2 * tid4;
          g[mt][nt][0] += bf16r(o[nt][0] + B.out_b[col]);
          g[mt][nt][1] += bf16r(o[nt][1] + B.out_b[col + 1]);
          g[mt][nt][2] += bf16r(o[nt][2] + B.out_b[col]);
          g[mt][nt][3] += bf16r(o[nt][3] + B.out_b[col + 1]);
        }
      }
    }
    // Final norm (fp32) and the features out: [token][card][width].
    float fin[2][4][4];
    grid_rms(g, S.final_norm, tid4, fin);
    float* base = cards + token * (kGCards * kGW);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int card = mt * 16 + gid + 8 * hf;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<float2*>(base + card * kGW + 8 * j + 2 * tid4) =
              make_float2(fin[mt][j][2 * hf], fin[mt][j][2 * hf + 1]);
      }
  }
}

}  // namespace
}  // namespace cg

extern "C" int cg_card_grid(const cg_card_grid_weights* weights, const void* codes, int codes_dtype, int64_t n,
                            int64_t codes_stride, float* cards, void* stream) {
  using namespace cg;
  CG_REQUIRE(weights, "cg_card_grid: NULL weights");
  const cg_card_grid_weights& w = *weights;
  CG_REQUIRE(w.width == kGW && w.hidden == kGH && w.kernel == 3,
             "cg_card_grid: card width %d, hidden %d and %d taps supported (got %d, %d, %d)", kGW, kGH, 3, w.width,
             w.hidden, w.kernel);
  CG_REQUIRE(w.blocks >= 0 && w.blocks <= kGMaxBlocks, "cg_card_grid: blocks must be 0..%d", kGMaxBlocks);
  CG_REQUIRE(w.codes >= 1 && w.codes <= kGMaxCodes, "cg_card_grid: code vocabulary must be 1..%d", kGMaxCodes);
  CG_REQUIRE(codes_dtype == CG_I16 || codes_dtype == CG_I32 || codes_dtype == CG_I64, "cg_card_grid: bad code dtype");
  CG_REQUIRE(n >= 0 && codes_stride >= kGCards, "cg_card_grid: bad count or code row stride");
  if (n == 0) return CG_OK;
  CG_REQUIRE(codes && cards && w.code_emb && w.rank_emb && w.final_norm, "cg_card_grid: NULL pointer");
  for (int b = 0; b < w.blocks; ++b)
    CG_REQUIRE(w.norm_w[b] && w.conv_w[b] && w.conv_b[b] && w.across_w[b] && w.out_w[b] && w.out_b[b],
               "cg_card_grid: NULL weight in block %d", b);
  const size_t smem = sizeof(GridSmem);
  static bool configured[64] = {false};
  int device = 0;
  cudaGetDevice(&device);
  if (!configured[device & 63]) {
    cudaError_t err =
        cudaFuncSetAttribute(card_grid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "card_grid_kernel smem: %s", cudaGetErrorString(err));
    configured[device & 63] = true;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, card_grid_kernel, kGridWarps * 32, smem);
  if (per_sm < 1) per_sm = 1;
  int64_t blocks = static_cast<int64_t>(sm_count()) * per_sm;
  const int64_t needed = (n + kGridWarps - 1) / kGridWarps;
  if (blocks > needed) blocks = needed;
  return launch_pdl("card_grid_kernel", card_grid_kernel, dim3(static_cast<unsigned>(blocks)), dim3(kGridWarps * 32),
                    smem, static_cast<cudaStream_t>(stream), w, codes, codes_dtype, n, codes_stride, cards);
}
