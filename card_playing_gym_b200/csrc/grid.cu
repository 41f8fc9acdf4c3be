// Card grids: per-card features of a token's card codes.
//
// Reference: cardgym/games/piquet/model.py:180-240 (`CardGrid.cards`), 129-177 (`GridBlock`),
// 118-126 (`GridNorm`): a 4 x 8 grid, a 3-tap zero-padded convolution along the ranks; and
// rummy's ledger grid, cardgym/games/rummy/model.py:112-225: a 4 x 13 grid, a 5-tap circular
// convolution. For one token, the grid (card = suit * ranks + rank) starts as
// code_emb[code] + rank_emb[rank] (fp32) and goes through `blocks` residual blocks:
//   rows   = RMSNorm(grid)                                     per card, over the width
//   along  = conv over ranks of rows, + bias                   cards x 64 hidden
//   across = (mean over suits of rows) @ W_across              ranks x 64 hidden
//   grid  += out(GELU(along + across[rank])) + bias            cards x 32 width
// then a final RMSNorm. The reference runs this under bf16 autocast in its rollouts: every
// Linear / matmul output (with its bias) is rounded to bf16, as are their sum and the GELU,
// while the residual grid and the norms stay fp32. This kernel computes exactly that form:
// bf16 tensor-core operands (mma.sync m16n8k16), fp32 accumulation, the same rounding points.
//
// One warp per token: the grid lives in registers in the MMA accumulator layout (m16 tiles of
// cards x four n8 tiles of width); the normalised rows go through shared memory once (padded
// ranks, zero or wrapped, so the convolution is one 32-wide k-block per tap of an m16n8k16
// GEMM read by ldmatrix); the GELU output feeds the output GEMM straight from registers.
// Weights sit in shared memory in bf16, [n][k] rows padded so ldmatrix rows hit distinct banks.
#include "common.cuh"

namespace cg {
namespace {

constexpr int kGridWarps = 8;
constexpr int kGW = 32;        // card width
constexpr int kGH = 64;        // block hidden width
constexpr int kGSuits = 4;
constexpr int kGMaxBlocks = 4;
constexpr int kAcrossStride = kGW + 8;   // bf16 per row (80 bytes)
constexpr int kOutStride = kGH + 8;      // 144 bytes
constexpr int kRowStride = kGW + 8;      // normed / pooled rows (80 bytes)
constexpr int kXStride = kGH + 8;        // per-warp across rows (144 bytes)

// kRanks ranks per suit (cards = 4 * kRanks, in m16 tiles), kTaps rank taps, circular or
// zero-padded rank ends.
template <int kRanks, int kTaps, bool kCircular>
struct GridShape {
  static constexpr int kCards = kGSuits * kRanks;
  static constexpr int kMT = (kCards + 15) / 16;          // m16 tiles of cards
  static constexpr int kHalf = kTaps / 2;
  static constexpr int kPadRanks = kRanks + 2 * kHalf;   // rows per suit in shared memory
  static constexpr int kConvK = kTaps * kGW;
  static constexpr int kConvStride = kConvK + 8;         // 208 (3 taps) or 336 (5 taps) bytes
};

template <typename G>
struct GridBlockSmem {
  __nv_bfloat16 conv[kGH * G::kConvStride];   // [hidden n][tap * 32 + width k]
  __nv_bfloat16 across[kGH * kAcrossStride];  // [hidden n][width k]
  __nv_bfloat16 out[kGW * kOutStride];        // [width n][hidden k]
  float norm[kGW];
  float conv_b[kGH];  // bf16-rounded (autocast casts the bias with the weight)
  float out_b[kGW];
};

template <typename G>
struct GridWarpSmem {
  __nv_bfloat16 normed[kGSuits * G::kPadRanks * kRowStride];  // padded ranks: zero or wrapped
  __nv_bfloat16 pooled[16 * kRowStride];                      // ranks; the rest zero
  __nv_bfloat16 across[16 * kXStride];                        // bf16 across rows per rank
};

template <typename G>
struct GridSmem {
  float rank[16 * kGW];
  float final_norm[kGW];
  GridBlockSmem<G> block[kGMaxBlocks];
  GridWarpSmem<G> warp[kGridWarps];
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

// RMSNorm of the rows this lane holds (rows gid and gid + 8 of each m16 tile) into `out`:
// a row's 32 values are spread over the four lanes of a quad.
template <int kMT>
__device__ __forceinline__ void grid_rms(const float (&g)[kMT][4][4], const float* weight, int tid4,
                                         float (&out)[kMT][4][4]) {
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt) {
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

template <int kRanks, int kTaps, bool kCircular>
__global__ void __launch_bounds__(kGridWarps * 32) card_grid_kernel(const cg_card_grid_weights w, const void* codes,
                                                                     int codes_dtype, int64_t n, int64_t stride,
                                                                     float* cards) {
  using G = GridShape<kRanks, kTaps, kCircular>;
  constexpr int kMT = G::kMT, kCards = G::kCards;
  extern __shared__ __align__(16) unsigned char grid_smem_raw[];
  GridSmem<G>& S = *reinterpret_cast<GridSmem<G>*>(grid_smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gid = lane >> 2, tid4 = lane & 3;
  const int nblocks = w.blocks;

  // Stage the weights (bf16 GEMM operands in [n][k] rows; fp32 norms, bf16-rounded biases).
  for (int i = tid; i < kRanks * kGW; i += blockDim.x) S.rank[i] = w.rank_emb[i];
  for (int i = tid; i < kGW; i += blockDim.x) S.final_norm[i] = w.final_norm[i];
  for (int b = 0; b < nblocks; ++b) {
    GridBlockSmem<G>& B = S.block[b];
    for (int i = tid; i < kGH * kGW * kTaps; i += blockDim.x) {  // conv weight [hidden][width][tap]
      const int hh = i / (kGW * kTaps), rem = i - hh * kGW * kTaps, wi = rem / kTaps, tap = rem - wi * kTaps;
      B.conv[hh * G::kConvStride + tap * kGW + wi] = __float2bfloat16_rn(w.conv_w[b][i]);
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
  // Zero the per-warp scratch once: padded ranks (zero-padded grids), pooled rows past kRanks.
  GridWarpSmem<G>& Wp = S.warp[warp];
  for (int i = lane; i < kGSuits * G::kPadRanks * kRowStride; i += 32) Wp.normed[i] = __float2bfloat16_rn(0.f);
  for (int i = lane; i < 16 * kRowStride; i += 32) Wp.pooled[i] = __float2bfloat16_rn(0.f);
  pdl_wait();
  pdl_trigger();
  __syncthreads();

  for (int64_t token = static_cast<int64_t>(blockIdx.x) * kGridWarps + warp; token < n;
       token += static_cast<int64_t>(gridDim.x) * kGridWarps) {
    // Card codes: lane c holds cards c and c + 32 (when there are more than 32 cards).
    int my_code[2] = {0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int card = lane + 32 * h;
      if (card < kCards) {
        int64_t code = grid_code(codes, codes_dtype, token * stride + card);
        if (code < 0 || code >= w.codes) {
          raise_fault(0x230);
          code = 0;
        }
        my_code[h] = static_cast<int>(code);
      }
    }
    // The grid in accumulator layout: g[mt][j][e] is card mt*16 + gid (+8 for e >= 2), width
    // column 8j + 2*tid4 (+1 for odd e). Rows past the last card stay zero.
    float g[kMT][4][4];
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int card = mt * 16 + gid + 8 * hf;
        const int src = card < kCards ? card : 0;
        const int c0 = __shfl_sync(0xffffffffu, my_code[0], src & 31);
        const int c1 = __shfl_sync(0xffffffffu, my_code[1], src & 31);
        const int c = src < 32 ? c0 : c1;
        const float* ce = w.code_emb + c * kGW;
        const float* re = S.rank + (src % kRanks) * kGW;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int col = 8 * j + 2 * tid4;
          const float2 cv = __ldg(reinterpret_cast<const float2*>(ce + col));
          g[mt][j][2 * hf] = card < kCards ? cv.x + re[col] : 0.f;
          g[mt][j][2 * hf + 1] = card < kCards ? cv.y + re[col + 1] : 0.f;
        }
      }

    for (int b = 0; b < nblocks; ++b) {
      const GridBlockSmem<G>& B = S.block[b];
      {
        float nm[kMT][4][4];
        grid_rms<kMT>(g, B.norm, tid4, nm);
        __syncwarp();  // the previous block's or token's reads of the scratch are done
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int card = mt * 16 + gid + 8 * hf;
            if (card >= kCards) continue;
            const int s = card / kRanks, r = card % kRanks;
            uint32_t v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) v[j] = pack_bf16(nm[mt][j][2 * hf], nm[mt][j][2 * hf + 1]);
            auto put = [&](int padded) {
              __nv_bfloat16* row = Wp.normed + (s * G::kPadRanks + padded) * kRowStride;
#pragma unroll
              for (int j = 0; j < 4; ++j) *reinterpret_cast<uint32_t*>(row + 8 * j + 2 * tid4) = v[j];
            };
            put(r + G::kHalf);
            if (kCircular) {  // the wrapped copies the convolution reads past either end
              if (r >= kRanks - G::kHalf) put(r + G::kHalf - kRanks);
              if (r < G::kHalf) put(r + G::kHalf + kRanks);
            }
          }
      }
      __syncwarp();
      // Suit means (the reference's [1, 4] matmul of 1/4: exact products, fp32 sums, one rounding).
      for (int idx = lane; idx < kRanks * 16; idx += 32) {
        const int r = idx >> 4, cp = idx & 15;
        float a = 0.f, c = 0.f;
#pragma unroll
        for (int s = 0; s < kGSuits; ++s) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(
              Wp.normed + (s * G::kPadRanks + r + G::kHalf) * kRowStride + 2 * cp));
          a = fmaf(0.25f, f.x, a);
          c = fmaf(0.25f, f.y, c);
        }
        *reinterpret_cast<uint32_t*>(Wp.pooled + r * kRowStride + 2 * cp) = pack_bf16(a, c);
      }
      __syncwarp();
      // Across-suit projection of the suit means (ranks x 64 hidden), rounded, to shared memory.
      {
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
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int col = 8 * nt + 2 * tid4;
          *reinterpret_cast<uint32_t*>(Wp.across + gid * kXStride + col) = pack_bf16(xs[nt][0], xs[nt][1]);
          *reinterpret_cast<uint32_t*>(Wp.across + (gid + 8) * kXStride + col) = pack_bf16(xs[nt][2], xs[nt][3]);
        }
      }
      __syncwarp();
      // Rank convolution, the sum with the across rows, GELU and the output layer, two m16
      // tiles of cards at a time (the grid updates do not feed this block's other tiles: their
      // normalised rows are already in shared memory).
#pragma unroll
      for (int p = 0; p < kMT; p += 2) {
        float acc[2][8][4];
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int nt = 0; nt < 8; ++nt) acc[m][nt][0] = acc[m][nt][1] = acc[m][nt][2] = acc[m][nt][3] = 0.f;
#pragma unroll
        for (int tap = 0; tap < kTaps; ++tap) {
#pragma unroll
          for (int kh = 0; kh < 2; ++kh) {
            uint32_t a[2][4];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
              int card = (p + m) * 16 + (lane & 15);
              if (card >= kCards) card = kCards - 1;  // padding rows: any finite row, never stored
              const int s = card / kRanks, r = card % kRanks;
              g_ldmatrix_x4(a[m][0], a[m][1], a[m][2], a[m][3],
                            gsmem(Wp.normed + (s * G::kPadRanks + r + tap) * kRowStride + kh * 16 + (lane >> 4) * 8));
            }
#pragma unroll
            for (int np = 0; np < 4; ++np) {
              uint32_t b0, b1, b2, b3;
              g_ldmatrix_x4(b0, b1, b2, b3,
                            gsmem(B.conv + (16 * np + (lane & 15)) * G::kConvStride + tap * kGW + kh * 16 +
                                  (lane >> 4) * 8));
#pragma unroll
              for (int m = 0; m < 2; ++m) {
                g_mma(acc[m][2 * np], a[m][0], a[m][1], a[m][2], a[m][3], b0, b2);
                g_mma(acc[m][2 * np + 1], a[m][0], a[m][1], a[m][2], a[m][3], b1, b3);
              }
            }
          }
        }
        // mixed = bf16(bf16(along + bias) + across[rank]); GELU rounded to bf16.
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int card = (p + m) * 16 + gid + 8 * hf;
            const int r = (card < kCards ? card : 0) % kRanks;
            const __nv_bfloat16* xr = Wp.across + r * kXStride;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
              const int col = 8 * nt + 2 * tid4;
              const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + col));
              float v0 = bf16r(bf16r(acc[m][nt][2 * hf] + B.conv_b[col]) + x.x);
              float v1 = bf16r(bf16r(acc[m][nt][2 * hf + 1] + B.conv_b[col + 1]) + x.y);
              v0 = 0.5f * v0 * (1.f + erff(v0 * 0.70710678118654752f));
              v1 = 0.5f * v1 * (1.f + erff(v1 * 0.70710678118654752f));
              acc[m][nt][2 * hf] = v0;
              acc[m][nt][2 * hf + 1] = v1;
            }
          }
        // Output layer from registers (accumulator pairs are the A fragments), + bias, rounded.
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          float o[4][4];
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a0 = pack_bf16(acc[m][2 * j][0], acc[m][2 * j][1]);
            const uint32_t a1 = pack_bf16(acc[m][2 * j][2], acc[m][2 * j][3]);
            const uint32_t a2 = pack_bf16(acc[m][2 * j + 1][0], acc[m][2 * j + 1][1]);
            const uint32_t a3 = pack_bf16(acc[m][2 * j + 1][2], acc[m][2 * j + 1][3]);
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
            g[p + m][nt][0] += bf16r(o[nt][0] + B.out_b[col]);
            g[p + m][nt][1] += bf16r(o[nt][1] + B.out_b[col + 1]);
            g[p + m][nt][2] += bf16r(o[nt][2] + B.out_b[col]);
            g[p + m][nt][3] += bf16r(o[nt][3] + B.out_b[col + 1]);
          }
        }
      }
    }
    // Final norm (fp32) and the features out: [token][card][width].
    float fin[kMT][4][4];
    grid_rms<kMT>(g, S.final_norm, tid4, fin);
    float* base = cards + token * (kCards * kGW);
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int card = mt * 16 + gid + 8 * hf;
        if (card >= kCards) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<float2*>(base + card * kGW + 8 * j + 2 * tid4) =
              make_float2(fin[mt][j][2 * hf], fin[mt][j][2 * hf + 1]);
      }
  }
}

template <int kRanks, int kTaps, bool kCircular>
int launch_grid(const cg_card_grid_weights& w, const void* codes, int codes_dtype, int64_t n, int64_t stride,
                float* cards, cudaStream_t s) {
  using G = GridShape<kRanks, kTaps, kCircular>;
  auto kernel = card_grid_kernel<kRanks, kTaps, kCircular>;
  const size_t smem = sizeof(GridSmem<G>);
  static bool configured[64] = {false};
  static int per_sm[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (!configured[device & 63]) {
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "card_grid_kernel smem: %s", cudaGetErrorString(err));
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[device & 63], kernel, kGridWarps * 32, smem);
    configured[device & 63] = true;
  }
  const int occupancy = per_sm[device & 63] > 0 ? per_sm[device & 63] : 1;
  int64_t blocks = static_cast<int64_t>(sm_count()) * occupancy;
  const int64_t needed = (n + kGridWarps - 1) / kGridWarps;
  if (blocks > needed) blocks = needed;
  return launch_pdl("card_grid_kernel", kernel, dim3(static_cast<unsigned>(blocks)), dim3(kGridWarps * 32), smem, s,
                    w, codes, codes_dtype, n, stride, cards);
}

}  // namespace
}  // namespace cg

extern "C" int cg_card_grid(const cg_card_grid_weights* weights, const void* codes, int codes_dtype, int64_t n,
                            int64_t codes_stride, float* cards, void* stream) {
  using namespace cg;
  CG_REQUIRE(weights, "cg_card_grid: NULL weights");
  const cg_card_grid_weights& w = *weights;
  CG_REQUIRE(w.width == kGW && w.hidden == kGH, "cg_card_grid: card width %d and hidden %d supported (got %d, %d)",
             kGW, kGH, w.width, w.hidden);
  const bool piquet = w.ranks == 8 && w.kernel == 3 && !w.circular;
  const bool rummy = w.ranks == 13 && w.kernel == 5 && w.circular;
  CG_REQUIRE(piquet || rummy,
             "cg_card_grid: grids of 8 ranks x 3 zero-padded taps (piquet) or 13 ranks x 5 circular taps (rummy)");
  CG_REQUIRE(w.blocks >= 0 && w.blocks <= kGMaxBlocks, "cg_card_grid: blocks must be 0..%d", kGMaxBlocks);
  CG_REQUIRE(w.codes >= 1, "cg_card_grid: empty code vocabulary");
  CG_REQUIRE(codes_dtype == CG_I16 || codes_dtype == CG_I32 || codes_dtype == CG_I64, "cg_card_grid: bad code dtype");
  CG_REQUIRE(n >= 0 && codes_stride >= 4 * w.ranks, "cg_card_grid: bad count or code row stride");
  if (n == 0) return CG_OK;
  CG_REQUIRE(codes && cards && w.code_emb && w.rank_emb && w.final_norm, "cg_card_grid: NULL pointer");
  CG_REQUIRE((reinterpret_cast<uintptr_t>(w.code_emb) & 7) == 0, "cg_card_grid: code table must be 8-byte aligned");
  for (int b = 0; b < w.blocks; ++b)
    CG_REQUIRE(w.norm_w[b] && w.conv_w[b] && w.conv_b[b] && w.across_w[b] && w.out_w[b] && w.out_b[b],
               "cg_card_grid: NULL weight in block %d", b);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (piquet) return launch_grid<8, 3, false>(w, codes, codes_dtype, n, codes_stride, cards, s);
  return launch_grid<13, 5, true>(w, codes, codes_dtype, n, codes_stride, cards, s);
}
