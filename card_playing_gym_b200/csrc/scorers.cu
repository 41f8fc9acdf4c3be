// Pointer heads: one logit per card of the readout state.
//
// Reference: cardgym/games/piquet/model.py:348-363 (`CardScorer.forward`):
//   mixed  = query(hidden)[:, None, :] + card(grid) + card_id.weight      [N, C, dim]
//   logits = out(GELU(hidden_layer(LayerNorm(mixed))))                    [N, C]
// (query: Linear d -> dim with bias; card: Linear card_width -> dim without; LayerNorm over
// dim, eps 1e-5; hidden_layer: Linear dim -> dim; exact-erf GELU; out: Linear dim -> 1), used
// by PiquetActor.policy_logits (model.py:399-411) for the exchange and play heads.
//
// One warp per decision, lane c = card c: the warp computes the query row once (lanes split
// its outputs), then every lane runs its card's whole chain in registers (the projection of
// its grid row, the LayerNorm over its own dim values, the hidden layer fused with GELU and
// the output dot), so no cross-lane reduction is needed. All weights sit in shared memory,
// transposed where lanes read different rows, and reach the lanes as broadcasts.
// Arithmetic is fp32 throughout (the grid may be fp32, bf16 or fp16).
//
// Candidate pointer head: cardgym/games/rummy/model.py:292-357 (`CandidateScorer.forward`),
// called by RummyActor.policy_logits (391-399) for the draw and play heads. Per candidate:
//   summed_s = counts_s @ grid   (slot 0: the cards it moves, 1: a lay-off's target meld,
//                                 2: the cards a draw takes from the pile, as counts)
//   candidate = Σ_s W_s summed_s + Σ_s counts_s @ id_s + kind_emb[kind] + size_emb[#cards]
//   logits = out(GELU(hidden(LayerNorm(query(h)[:, None] + candidate))))
// One warp per decision (its grid rows staged in shared memory, padded so lanes gathering
// different cards hit different banks), lane = candidate. The slot sums are formed first and
// projected once, as the reference does by linearity. Sums are fp32; their order differs from
// the reference's GEMMs only in rounding.
#include "common.cuh"

namespace cg {
namespace {

constexpr int kScorerWarps = 8;
constexpr int kScorerDim = 64;    // score_dim (the reference's default; the kernel is specialised on it)
constexpr int kScorerMaxWidth = 32;  // card_width (piquet: 32)
constexpr int kScorerMaxD = 512;

struct ScorerSmem {
  // Offsets (floats) inside the dynamic shared memory.
  int qT, cw, idT, nw, nb, hw, hb, ow, h, q, total;
};

__host__ __device__ inline ScorerSmem scorer_smem(int d, int width, int cards) {
  ScorerSmem s{};
  int at = 0;
  s.qT = at, at += d * kScorerDim;           // query weight transposed [d][dim]
  s.cw = at, at += kScorerDim * width;       // card weight transposed [width][dim]
  s.idT = at, at += kScorerDim * 32;         // card ids transposed [dim][32] (cards <= 32, zero-padded)
  s.nw = at, at += kScorerDim;
  s.nb = at, at += kScorerDim;
  s.hw = at, at += kScorerDim * kScorerDim;  // hidden weight transposed [in][out]
  s.hb = at, at += kScorerDim;
  s.ow = at, at += kScorerDim;
  s.h = at, at += kScorerWarps * d;          // per-warp hidden row
  s.q = at, at += kScorerWarps * kScorerDim;  // per-warp query row
  s.total = at;
  (void)cards;
  return s;
}

__device__ __forceinline__ float scorer_load(const void* p, int dtype, int64_t i) {
  if (dtype == CG_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == CG_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

__device__ __forceinline__ float scorer_gelu(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752f)); }

// m[o] += sum_j W[o][j] x[j] (in j order) with W staged transposed, WT[j][o]: each j is 16
// broadcast float4 reads feeding the 64 independent accumulators.
template <int kW>
__device__ __forceinline__ void project_add(const float* WT, const float (&x)[kW], int width, float (&m)[kScorerDim]) {
#pragma unroll
  for (int j = 0; j < kW; ++j) {
    if (j < width) {
      const float xj = x[j];
#pragma unroll
      for (int o = 0; o < kScorerDim; o += 4) {
        const float4 wv = *reinterpret_cast<const float4*>(WT + j * kScorerDim + o);
        m[o] = fmaf(wv.x, xj, m[o]);
        m[o + 1] = fmaf(wv.y, xj, m[o + 1]);
        m[o + 2] = fmaf(wv.z, xj, m[o + 2]);
        m[o + 3] = fmaf(wv.w, xj, m[o + 3]);
      }
    }
  }
}

// LayerNorm over the dim values in place (two passes, fp32, eps 1e-5).
__device__ __forceinline__ void scorer_layer_norm(float (&m)[kScorerDim], const float* nw, const float* nb) {
  float mean = 0.f;
#pragma unroll
  for (int o = 0; o < kScorerDim; ++o) mean += m[o];
  mean *= 1.f / kScorerDim;
  float var = 0.f;
#pragma unroll
  for (int o = 0; o < kScorerDim; ++o) {
    const float t = m[o] - mean;
    var = fmaf(t, t, var);
  }
  const float rstd = rsqrtf(var * (1.f / kScorerDim) + 1e-5f);
#pragma unroll
  for (int o = 0; o < kScorerDim; ++o) m[o] = (m[o] - mean) * rstd * nw[o] + nb[o];
}

// out(GELU(hidden(m))) with the hidden weight staged transposed (hwT[k][o]): sixteen hidden
// units at a time, each summed over k in order; the output dot in unit order.
__device__ __forceinline__ float scorer_head(const float (&m)[kScorerDim], const float* hwT, const float* hb,
                                             const float* ow) {
  float out = 0.f;
#pragma unroll 1
  for (int o0 = 0; o0 < kScorerDim; o0 += 16) {
    float h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) h[j] = 0.f;
#pragma unroll
    for (int k = 0; k < kScorerDim; ++k) {
      const float mk = m[k];
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const float4 wv = *reinterpret_cast<const float4*>(hwT + k * kScorerDim + o0 + j);
        h[j] = fmaf(wv.x, mk, h[j]);
        h[j + 1] = fmaf(wv.y, mk, h[j + 1]);
        h[j + 2] = fmaf(wv.z, mk, h[j + 2]);
        h[j + 3] = fmaf(wv.w, mk, h[j + 3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) out = fmaf(ow[o0 + j], scorer_gelu(h[j] + hb[o0 + j]), out);
  }
  return out;
}

// The query row of one decision: lanes own outputs lane and lane + 32, four partial sums each.
__device__ __forceinline__ void scorer_query(const float* qT, const float* hrow, int d, const float* bias, int lane,
                                             float* qrow) {
  float a[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  int k = 0;
  for (; k + 4 <= d; k += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float hk = hrow[k + u];
      a[0][u] = fmaf(qT[(k + u) * kScorerDim + lane], hk, a[0][u]);
      a[1][u] = fmaf(qT[(k + u) * kScorerDim + lane + 32], hk, a[1][u]);
    }
  }
  for (; k < d; ++k) {
    a[0][0] = fmaf(qT[k * kScorerDim + lane], hrow[k], a[0][0]);
    a[1][0] = fmaf(qT[k * kScorerDim + lane + 32], hrow[k], a[1][0]);
  }
  qrow[lane] = bias[lane] + ((a[0][0] + a[0][1]) + (a[0][2] + a[0][3]));
  qrow[lane + 32] = bias[lane + 32] + ((a[1][0] + a[1][1]) + (a[1][2] + a[1][3]));
}

__global__ void __launch_bounds__(kScorerWarps * 32) card_scorer_kernel(const cg_card_scorer_weights w, const float* hidden,
                                                                         int64_t n, const void* grid, int grid_dtype,
                                                                         float* logits) {
  extern __shared__ __align__(16) float sc_smem[];
  const int d = w.d_model, width = w.card_width, cards = w.cards;
  const ScorerSmem L = scorer_smem(d, width, cards);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // Stage the weights (constant over the launch).
  for (int i = tid; i < kScorerDim * d; i += blockDim.x) {
    const int o = i / d, k = i - o * d;
    sc_smem[L.qT + k * kScorerDim + o] = w.query_w[i];
  }
  for (int i = tid; i < kScorerDim * width; i += blockDim.x) {
    const int o = i / width, j = i - o * width;
    sc_smem[L.cw + j * kScorerDim + o] = w.card_w[i];  // transposed [width][dim]
  }
  for (int i = tid; i < kScorerDim * 32; i += blockDim.x) {
    const int o = i / 32, c = i - o * 32;
    sc_smem[L.idT + i] = c < cards ? w.card_id[c * kScorerDim + o] : 0.f;
  }
  for (int i = tid; i < kScorerDim; i += blockDim.x) {
    sc_smem[L.nw + i] = w.norm_w[i];
    sc_smem[L.nb + i] = w.norm_b[i];
    sc_smem[L.hb + i] = w.hidden_b[i];
    sc_smem[L.ow + i] = w.out_w[i];
  }
  for (int i = tid; i < kScorerDim * kScorerDim; i += blockDim.x) {
    const int o = i / kScorerDim, k = i - o * kScorerDim;
    sc_smem[L.hw + k * kScorerDim + o] = w.hidden_w[i];  // transposed [k][o]
  }
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const float out_b = *w.out_b;
  float* hrow = sc_smem + L.h + warp * d;
  float* qrow = sc_smem + L.q + warp * kScorerDim;

  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kScorerWarps + warp; i < n;
       i += static_cast<int64_t>(gridDim.x) * kScorerWarps) {
    __syncwarp();
    for (int k = lane; k < d; k += 32) hrow[k] = hidden[i * d + k];
    __syncwarp();
    scorer_query(sc_smem + L.qT, hrow, d, w.query_b, lane, qrow);
    __syncwarp();

    const bool live = lane < cards;
    const int c = live ? lane : 0;
    float g[kScorerMaxWidth];
    const int64_t gbase = (i * cards + c) * width;
#pragma unroll
    for (int k = 0; k < kScorerMaxWidth; ++k) g[k] = k < width ? scorer_load(grid, grid_dtype, gbase + k) : 0.f;
    // mixed = query + card(grid) + card_id, the reference's order of the two adds.
    float m[kScorerDim];
#pragma unroll
    for (int o = 0; o < kScorerDim; ++o) m[o] = 0.f;
    project_add(sc_smem + L.cw, g, width, m);
#pragma unroll
    for (int o = 0; o < kScorerDim; ++o) m[o] = (qrow[o] + m[o]) + sc_smem[L.idT + o * 32 + c];
    scorer_layer_norm(m, sc_smem + L.nw, sc_smem + L.nb);
    const float out = scorer_head(m, sc_smem + L.hw, sc_smem + L.hb, sc_smem + L.ow);
    if (live) logits[i * cards + lane] = out + out_b;
  }
}

constexpr int kCandWarps = 6;
constexpr int kCandMaxCards = 64;  // card types (rummy: 52)
constexpr int kCandMaxList = 16;   // cards per slot list (rummy: MAX_MELD_CARDS = 13)

struct CandSmem {
  int qT, w, idT, kindT, sizeT, nw, nb, hw, hb, ow, grid, h, q, total;
  int cpad, gpad;
};

__host__ __device__ inline CandSmem cand_smem(const cg_candidate_scorer_weights& w) {
  CandSmem s{};
  s.cpad = w.cards | 1;         // odd row stride of the transposed id tables
  s.gpad = w.card_width + 1;    // odd row stride of the staged grid rows
  int at = 0;
  s.qT = at, at += w.d_model * kScorerDim;
  s.w = at, at += 3 * kScorerDim * w.card_width;  // card, target, taken projections [3][width][dim]
  s.idT = at, at += 3 * kScorerDim * s.cpad;      // card, target, taken ids transposed [3][dim][cards]
  s.kindT = at, at += kScorerDim * w.kinds;
  s.sizeT = at, at += kScorerDim * w.sizes;
  s.nw = at, at += kScorerDim;
  s.nb = at, at += kScorerDim;
  s.hw = at, at += kScorerDim * kScorerDim;
  s.hb = at, at += kScorerDim;
  s.ow = at, at += kScorerDim;
  s.grid = at, at += kCandWarps * w.cards * s.gpad;
  s.h = at, at += kCandWarps * w.d_model;
  s.q = at, at += kCandWarps * kScorerDim;
  s.total = at;
  return s;
}

__global__ void __launch_bounds__(kCandWarps * 32) candidate_scorer_kernel(
    const cg_candidate_scorer_weights w, const float* hidden, int64_t n, int k_cands, int list, const void* grid,
    int grid_dtype, const int64_t* kind, const int64_t* cards, const int64_t* target, const float* taken,
    float* logits) {
  extern __shared__ __align__(16) float cs_smem[];
  const CandSmem L = cand_smem(w);
  const int d = w.d_model, width = w.card_width, ncards = w.cards;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kScorerDim * d; i += blockDim.x) {
    const int o = i / d, k = i - o * d;
    cs_smem[L.qT + k * kScorerDim + o] = w.query_w[i];
  }
  const float* projections[3] = {w.card_w, w.target_w, w.taken_w};
  const float* identities[3] = {w.card_id, w.target_id, w.taken_id};
  for (int sl = 0; sl < 3; ++sl) {
    for (int i = tid; i < kScorerDim * width; i += blockDim.x) {
      const int o = i / width, j = i - o * width;
      cs_smem[L.w + sl * kScorerDim * width + j * kScorerDim + o] = projections[sl][i];  // [width][dim]
    }
    for (int i = tid; i < kScorerDim * ncards; i += blockDim.x) {
      const int c = i / kScorerDim, o = i - c * kScorerDim;
      cs_smem[L.idT + (sl * kScorerDim + o) * L.cpad + c] = identities[sl][i];
    }
  }
  for (int i = tid; i < kScorerDim * w.kinds; i += blockDim.x) {
    const int r = i / kScorerDim, o = i - r * kScorerDim;
    cs_smem[L.kindT + o * w.kinds + r] = w.kind_emb[i];
  }
  for (int i = tid; i < kScorerDim * w.sizes; i += blockDim.x) {
    const int r = i / kScorerDim, o = i - r * kScorerDim;
    cs_smem[L.sizeT + o * w.sizes + r] = w.size_emb[i];
  }
  for (int i = tid; i < kScorerDim; i += blockDim.x) {
    cs_smem[L.nw + i] = w.norm_w[i];
    cs_smem[L.nb + i] = w.norm_b[i];
    cs_smem[L.hb + i] = w.hidden_b[i];
    cs_smem[L.ow + i] = w.out_w[i];
  }
  for (int i = tid; i < kScorerDim * kScorerDim; i += blockDim.x) {
    const int o = i / kScorerDim, k = i - o * kScorerDim;
    cs_smem[L.hw + k * kScorerDim + o] = w.hidden_w[i];  // transposed [k][o]
  }
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  const float out_b = *w.out_b;
  float* grid_s = cs_smem + L.grid + warp * ncards * L.gpad;
  float* hrow = cs_smem + L.h + warp * d;
  float* qrow = cs_smem + L.q + warp * kScorerDim;
  const int no_card = ncards;

  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kCandWarps + warp; i < n;
       i += static_cast<int64_t>(gridDim.x) * kCandWarps) {
    __syncwarp();
    for (int x = lane; x < d; x += 32) hrow[x] = hidden[i * d + x];
    for (int x = lane; x < ncards * width; x += 32) {
      const int c = x / width, j = x - c * width;
      grid_s[c * L.gpad + j] = scorer_load(grid, grid_dtype, i * ncards * width + x);
    }
    __syncwarp();
    scorer_query(cs_smem + L.qT, hrow, d, w.query_b, lane, qrow);
    __syncwarp();

    for (int c0 = 0; c0 < k_cands; c0 += 32) {
      const int cand = c0 + lane;
      const bool live = cand < k_cands;
      const int64_t row = i * k_cands + (live ? cand : 0);
      float m[kScorerDim];
#pragma unroll
      for (int o = 0; o < kScorerDim; ++o) m[o] = 0.f;
      int size = 0;
      // Slots 0 (cards) and 1 (target): the listed cards, NO_CARD entries skipped.
#pragma unroll 1
      for (int sl = 0; sl < 2; ++sl) {
        const int64_t* ids = (sl == 0 ? cards : target) + row * list;
        float acc[kScorerMaxWidth];
#pragma unroll
        for (int j = 0; j < kScorerMaxWidth; ++j) acc[j] = 0.f;
        const float* idT = cs_smem + L.idT + sl * kScorerDim * L.cpad;
        float idacc[kScorerDim];
#pragma unroll
        for (int o = 0; o < kScorerDim; ++o) idacc[o] = 0.f;
        for (int e = 0; e < list; ++e) {
          const int64_t id = live ? ids[e] : no_card;
          if (id == no_card) continue;
          if (id < 0 || id > no_card) {
            raise_fault(0x220);
            continue;
          }
          size += sl == 0;
          const float* g = grid_s + id * L.gpad;
#pragma unroll
          for (int j = 0; j < kScorerMaxWidth; ++j)
            if (j < width) acc[j] += g[j];
#pragma unroll
          for (int o = 0; o < kScorerDim; ++o) idacc[o] += idT[o * L.cpad + id];
        }
        project_add(cs_smem + L.w + sl * kScorerDim * width, acc, width, m);
#pragma unroll
        for (int o = 0; o < kScorerDim; ++o) m[o] += idacc[o];
      }
      // Slot 2: the taken counts, dense over the card types.
      if (taken) {
        float acc[kScorerMaxWidth];
#pragma unroll
        for (int j = 0; j < kScorerMaxWidth; ++j) acc[j] = 0.f;
        const float* idT = cs_smem + L.idT + 2 * kScorerDim * L.cpad;
        float idacc[kScorerDim];
#pragma unroll
        for (int o = 0; o < kScorerDim; ++o) idacc[o] = 0.f;
        for (int c = 0; c < ncards; ++c) {
          const float t = live ? taken[row * ncards + c] : 0.f;
          if (t == 0.f) continue;
          const float* g = grid_s + c * L.gpad;
#pragma unroll
          for (int j = 0; j < kScorerMaxWidth; ++j)
            if (j < width) acc[j] = fmaf(t, g[j], acc[j]);
#pragma unroll
          for (int o = 0; o < kScorerDim; ++o) idacc[o] = fmaf(t, idT[o * L.cpad + c], idacc[o]);
        }
        project_add(cs_smem + L.w + 2 * kScorerDim * width, acc, width, m);
#pragma unroll
        for (int o = 0; o < kScorerDim; ++o) m[o] += idacc[o];
      }
      int kd = live ? static_cast<int>(kind[row]) : 0;
      if (kd < 0 || kd >= w.kinds) {
        raise_fault(0x221);
        kd = 0;
      }
      if (size >= w.sizes) {
        raise_fault(0x222);
        size = 0;
      }
#pragma unroll
      for (int o = 0; o < kScorerDim; ++o)
        m[o] = qrow[o] + ((m[o] + cs_smem[L.kindT + o * w.kinds + kd]) + cs_smem[L.sizeT + o * w.sizes + size]);
      scorer_layer_norm(m, cs_smem + L.nw, cs_smem + L.nb);
      const float out = scorer_head(m, cs_smem + L.hw, cs_smem + L.hb, cs_smem + L.ow);
      if (live) logits[row] = out + out_b;
    }
  }
}

}  // namespace
}  // namespace cg

extern "C" int cg_candidate_scorer(const cg_candidate_scorer_weights* weights, const float* hidden, int64_t n,
                                   int candidates, int list, const void* grid, int grid_dtype, const int64_t* kind,
                                   const int64_t* cards, const int64_t* target, const float* taken, float* logits,
                                   void* stream) {
  using namespace cg;
  CG_REQUIRE(weights, "cg_candidate_scorer: NULL weights");
  const cg_candidate_scorer_weights& w = *weights;
  CG_REQUIRE(w.dim == kScorerDim, "cg_candidate_scorer: score dim must be %d (got %d)", kScorerDim, w.dim);
  CG_REQUIRE(w.cards >= 1 && w.cards <= kCandMaxCards, "cg_candidate_scorer: cards must be 1..%d", kCandMaxCards);
  CG_REQUIRE(w.card_width >= 1 && w.card_width <= kScorerMaxWidth, "cg_candidate_scorer: card width must be 1..%d",
             kScorerMaxWidth);
  CG_REQUIRE(w.d_model >= 1 && w.d_model <= kScorerMaxD, "cg_candidate_scorer: d_model must be 1..%d", kScorerMaxD);
  CG_REQUIRE(w.kinds >= 1 && w.sizes >= 1, "cg_candidate_scorer: empty kind or size table");
  CG_REQUIRE(candidates >= 1 && list >= 0 && list <= kCandMaxList,
             "cg_candidate_scorer: candidates must be >= 1 and lists 0..%d cards", kCandMaxList);
  CG_REQUIRE(grid_dtype == CG_F32 || grid_dtype == CG_BF16 || grid_dtype == CG_F16,
             "cg_candidate_scorer: bad grid dtype");
  CG_REQUIRE(n >= 0, "cg_candidate_scorer: bad count");
  if (n == 0) return CG_OK;
  CG_REQUIRE(hidden && grid && logits && kind && cards && target, "cg_candidate_scorer: NULL input");
  CG_REQUIRE(w.query_w && w.query_b && w.card_w && w.target_w && w.taken_w && w.card_id && w.target_id &&
                 w.taken_id && w.kind_emb && w.size_emb && w.norm_w && w.norm_b && w.hidden_w && w.hidden_b &&
                 w.out_w && w.out_b,
             "cg_candidate_scorer: NULL weight");
  const CandSmem L = cand_smem(w);
  const size_t smem = static_cast<size_t>(L.total) * 4;
  CG_REQUIRE(smem <= 227 * 1024, "cg_candidate_scorer: weights need %zu bytes of shared memory", smem);
  static size_t configured[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (configured[device & 63] < smem) {
    cudaError_t err = cudaFuncSetAttribute(candidate_scorer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess)
      return set_error(CG_ERR_CUDA, "candidate_scorer_kernel smem: %s", cudaGetErrorString(err));
    configured[device & 63] = smem;
  }
  int64_t blocks = sm_count();
  const int64_t needed = (n + kCandWarps - 1) / kCandWarps;
  if (blocks > needed) blocks = needed;
  return launch_pdl("candidate_scorer_kernel", candidate_scorer_kernel, dim3(static_cast<unsigned>(blocks)),
                    dim3(kCandWarps * 32), smem, static_cast<cudaStream_t>(stream), w, hidden, n, candidates, list,
                    grid, grid_dtype, kind, cards, target, taken, logits);
}

extern "C" int cg_card_scorer(const cg_card_scorer_weights* weights, const float* hidden, int64_t n, const void* grid,
                              int grid_dtype, float* logits, void* stream) {
  using namespace cg;
  CG_REQUIRE(weights, "cg_card_scorer: NULL weights");
  const cg_card_scorer_weights& w = *weights;
  CG_REQUIRE(w.dim == kScorerDim, "cg_card_scorer: score dim must be %d (got %d)", kScorerDim, w.dim);
  CG_REQUIRE(w.cards >= 1 && w.cards <= 32, "cg_card_scorer: cards must be 1..32 (got %d)", w.cards);
  CG_REQUIRE(w.card_width >= 1 && w.card_width <= kScorerMaxWidth, "cg_card_scorer: card width must be 1..%d",
             kScorerMaxWidth);
  CG_REQUIRE(w.d_model >= 1 && w.d_model <= kScorerMaxD, "cg_card_scorer: d_model must be 1..%d", kScorerMaxD);
  CG_REQUIRE(grid_dtype == CG_F32 || grid_dtype == CG_BF16 || grid_dtype == CG_F16, "cg_card_scorer: bad grid dtype");
  CG_REQUIRE(n >= 0, "cg_card_scorer: bad count");
  if (n == 0) return CG_OK;
  CG_REQUIRE(hidden && grid && logits && w.query_w && w.query_b && w.card_w && w.card_id && w.norm_w && w.norm_b &&
                 w.hidden_w && w.hidden_b && w.out_w && w.out_b,
             "cg_card_scorer: NULL pointer");
  const ScorerSmem L = scorer_smem(w.d_model, w.card_width, w.cards);
  const size_t smem = static_cast<size_t>(L.total) * 4;
  CG_REQUIRE(smem <= 227 * 1024, "cg_card_scorer: weights need %zu bytes of shared memory", smem);
  static size_t configured[64] = {0};
  int device = 0;
  cudaGetDevice(&device);
  if (configured[device & 63] < smem) {
    cudaError_t err = cudaFuncSetAttribute(card_scorer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
    if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "card_scorer_kernel smem: %s", cudaGetErrorString(err));
    configured[device & 63] = smem;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, card_scorer_kernel, kScorerWarps * 32, smem);
  if (per_sm < 1) per_sm = 1;
  int64_t blocks = static_cast<int64_t>(sm_count()) * per_sm;
  const int64_t needed = (n + kScorerWarps - 1) / kScorerWarps;
  if (blocks > needed) blocks = needed;
  return launch_pdl("card_scorer_kernel", card_scorer_kernel, dim3(static_cast<unsigned>(blocks)),
                    dim3(kScorerWarps * 32), smem, static_cast<cudaStream_t>(stream), w, hidden, n, grid, grid_dtype,
                    logits);
}
