// Plump field lookup and the token-level ragged forward.
//
// Reference: cardgym/games/plump/model.py:94-167 (PlumpEmbedding: three embedding_bag
// sums + the NA-pattern row + the remaining-hand rank/suit rows on TRICK_WIN tokens)
// and cardgym/nn/model.py:76-89 (SequenceModel.forward_ragged = embed -> condition ->
// Trunk.forward_ragged). One fused lookup reads a packed [field rows + pattern rows,
// d | ple | value] table, so all three sums come from one pass over each token, with
// no boolean-mask nonzero (the reference's host sync, model.py:143).
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
constexpr int64_t kAlign = 256;
inline int64_t align_up(int64_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

__device__ __forceinline__ int64_t token_at(const void* tokens, int dtype, int64_t index) {
  if (dtype == CG_I16) return static_cast<const int16_t*>(tokens)[index];
  if (dtype == CG_I32) return static_cast<const int32_t*>(tokens)[index];
  return static_cast<const int64_t*>(tokens)[index];
}
}  // namespace

// One warp per token; lanes own 4 consecutive columns per 128-column block.
__global__ void __launch_bounds__(256) plump_embed_kernel(cg_plump_schema sc, const float* __restrict__ table, int width,
                                                          const void* __restrict__ tokens, int token_dtype, int64_t n,
                                                          float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t tok = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (tok >= n) return;
  const int64_t base = tok * sc.token_width;
  const int total_rows = sc.field_rows + sc.pattern_rows;
  // Resolve the row ids once per token (lane f holds field f; lanes 0..2*hand_slots-1 the hand rows).
  int field_row = -1;
  if (lane < sc.field_count) {
    const int64_t id = token_at(tokens, token_dtype, base + sc.field_slots[lane]);
    const bool present = sc.field_na[lane] < 0 || id != sc.field_na[lane];
    const int64_t row = id + sc.field_offsets[lane];
    if (present) {
      if (id < 0 || row >= sc.field_rows) {
        raise_fault(0x200);
      } else {
        field_row = static_cast<int>(row);
      }
    }
  }
  int64_t pattern = token_at(tokens, token_dtype, base + sc.slot_pattern);
  if (pattern < 0 || pattern >= sc.pattern_rows) {
    raise_fault(0x201);
    pattern = 0;
  }
  const bool trick_win = token_at(tokens, token_dtype, base + sc.slot_type) == sc.trick_win_type;
  int hand_row = -1;  // lane 2c: rank row of card c, lane 2c+1: its suit row
  if (trick_win && lane < 2 * sc.hand_slots) {
    const int64_t card = token_at(tokens, token_dtype, base + sc.slot_hand + lane / 2);
    if (card >= 0 && card < sc.num_cards) {
      hand_row = (lane & 1) ? static_cast<int>(card / sc.num_ranks) + sc.suit_offset
                            : static_cast<int>(card % sc.num_ranks) + sc.rank_offset;
    }
  }
  const bool vec = (width & 3) == 0;
  for (int c0 = 0; c0 < width; c0 += 128) {
    const int c = c0 + lane * 4;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float hand[4] = {0.f, 0.f, 0.f, 0.f};
    auto add_row = [&](float (&dst)[4], int row) {
      const float* src = table + static_cast<int64_t>(row) * width + c;
      if (vec && c + 3 < width) {
        const float4 v = *reinterpret_cast<const float4*>(src);
        dst[0] += v.x;
        dst[1] += v.y;
        dst[2] += v.z;
        dst[3] += v.w;
      } else {
        for (int j = 0; j < 4; ++j)
          if (c + j < width) dst[j] += src[j];
      }
    };
    for (int f = 0; f < sc.field_count; ++f) {
      const int row = __shfl_sync(0xffffffffu, field_row, f);
      if (row >= 0 && c < width) add_row(acc, row);
    }
    if (c < width) add_row(acc, sc.field_rows + static_cast<int>(pattern));
    if (trick_win) {
      for (int j = 0; j < 2 * sc.hand_slots; ++j) {
        const int row = __shfl_sync(0xffffffffu, hand_row, j);
        if (row >= 0 && c < width) add_row(hand, row);
      }
      for (int j = 0; j < 4; ++j) acc[j] += hand[j];
    }
    float* dst = out + tok * width + c;
    if (vec && c + 3 < width) {
      *reinterpret_cast<float4*>(dst) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    } else {
      for (int j = 0; j < 4; ++j)
        if (c + j < width) dst[j] = acc[j];
    }
  }
  (void)total_rows;
}

// ---- the lookup with table slices in shared memory ---------------------------------------------
// A token sums ~16-35 table rows of `width` floats; read from L2 that is ~145 KB per token.
// Here a CTA takes a block of tokens, resolves their row ids once into shared memory, then
// streams the table through shared memory in slices of kSliceF4 float4 columns (two slices
// in flight), so every row read of the sums is a shared-memory read. Sums run in the same
// order as plump_embed_kernel (fields, pattern, then the hand rows as one partial sum).
constexpr int kEmbedThreads = 512;
constexpr int kEmbedMaxTokens = 256;   // tokens per CTA
constexpr int kEmbedMain = 17;         // id slots: up to 16 fields + the pattern row
constexpr int kEmbedIds = kEmbedMain + 32;

struct EmbedIds {
  int16_t row[kEmbedIds];  // [0, n_main): fields then pattern; [kEmbedMain, +n_hand): hand rows
  uint8_t n_main, n_hand;
};



// Shared memory of a sliced lookup CTA: two table slices, the row ids and the token rows.
__host__ __device__ inline size_t embed_smem_bytes(int total_rows, int slice_f4, int tokens, int token_width) {
  return 2 * static_cast<size_t>(total_rows) * slice_f4 * 16 + static_cast<size_t>(tokens) * sizeof(EmbedIds) +
         (static_cast<size_t>(tokens) * token_width * 4 + 15) / 16 * 16;
}

// Grid: x = token blocks of tokens_per_cta, y = column groups of slices_per_cta slices (the
// split keeps every CTA's token passes full when the tokens alone would leave the last
// pass of each CTA partly idle).
template <int kSliceF4>  // float4 columns per slice = lanes per token
__global__ void __launch_bounds__(kEmbedThreads, 1) plump_embed_sliced_kernel(
    cg_plump_schema sc, const float* __restrict__ table, int width, const void* __restrict__ tokens, int token_dtype,
    int64_t n, int tokens_per_cta, int slices_per_cta, EmbedOut out) {
  extern __shared__ __align__(16) unsigned char emb_smem[];
  const int total_rows = sc.field_rows + sc.pattern_rows;
  float4* slices = reinterpret_cast<float4*>(emb_smem);  // [2][total_rows][kSliceF4]
  EmbedIds* ids = reinterpret_cast<EmbedIds*>(slices + 2 * total_rows * kSliceF4);
  int* tok_s = reinterpret_cast<int*>(ids + tokens_per_cta);  // [count][token_width], clamped to int32
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * tokens_per_cta;
  const int count = static_cast<int>(n - first < tokens_per_cta ? n - first : tokens_per_cta);
  const int width4 = width / 4;
  const int n_slices = (width4 + kSliceF4 - 1) / kSliceF4;
  const int s_begin = blockIdx.y * slices_per_cta;
  const int s_end = min(n_slices, s_begin + slices_per_cta);

  auto load_slice = [&](int slice, int buf) {
    const int c0 = slice * kSliceF4;
    float4* dst = slices + buf * total_rows * kSliceF4;
    for (int i = tid; i < total_rows * kSliceF4; i += kEmbedThreads) {
      const int r = i / kSliceF4, c = c0 + (i - r * kSliceF4);
      const bool valid = c < width4;
      const float4* src = reinterpret_cast<const float4*>(table + static_cast<int64_t>(r) * width) + (valid ? c : 0);
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                       static_cast<uint32_t>(__cvta_generic_to_shared(dst + i))),
                   "l"(src), "r"(valid ? 16 : 0)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (s_begin < s_end) load_slice(s_begin, 0);  // the table is constant: it loads while the kernel before finishes
  pdl_wait();
  pdl_trigger();
  if (s_begin >= s_end) return;

  // The CTA's token rows in one coalesced pass. Values are clamped to the int32 range, which
  // keeps every range check below (ids, patterns, cards) deciding as on the full value.
  {
    const int64_t base = first * sc.token_width;
    const int total = count * sc.token_width;
    for (int i = tid; i < total; i += kEmbedThreads) {
      const int64_t v = token_at(tokens, token_dtype, base + i);
      tok_s[i] = static_cast<int>(v < INT32_MIN ? INT32_MIN : (v > INT32_MAX ? INT32_MAX : v));
    }
  }
  __syncthreads();

  // Row ids, one warp per token (the same resolution as plump_embed_kernel).
  const unsigned lt = (1u << lane) - 1u;
  for (int t = warp; t < count; t += kEmbedThreads / 32) {
    const int* tok = tok_s + t * sc.token_width;
    int field_row = -1;
    if (lane < sc.field_count) {
      const int64_t id = tok[sc.field_slots[lane]];
      const bool present = sc.field_na[lane] < 0 || id != sc.field_na[lane];
      const int64_t row = id + sc.field_offsets[lane];
      if (present) {
        if (id < 0 || row >= sc.field_rows) {
          raise_fault(0x200);
        } else {
          field_row = static_cast<int>(row);
        }
      }
    }
    int64_t pattern = tok[sc.slot_pattern];
    if (pattern < 0 || pattern >= sc.pattern_rows) {
      if (lane == 0) raise_fault(0x201);
      pattern = 0;
    }
    const bool trick_win = tok[sc.slot_type] == sc.trick_win_type;
    int hand_row = -1;
    if (trick_win && lane < 2 * sc.hand_slots) {
      const int64_t card = tok[sc.slot_hand + lane / 2];
      if (card >= 0 && card < sc.num_cards) {
        hand_row = (lane & 1) ? static_cast<int>(card / sc.num_ranks) + sc.suit_offset
                              : static_cast<int>(card % sc.num_ranks) + sc.rank_offset;
      }
    }
    const unsigned fields = __ballot_sync(0xffffffffu, field_row >= 0);
    const unsigned hands = __ballot_sync(0xffffffffu, hand_row >= 0);
    EmbedIds& e = ids[t];
    if (field_row >= 0) e.row[__popc(fields & lt)] = static_cast<int16_t>(field_row);
    if (hand_row >= 0) e.row[kEmbedMain + __popc(hands & lt)] = static_cast<int16_t>(hand_row);
    if (lane == 0) {
      const int nf = __popc(fields);
      e.row[nf] = static_cast<int16_t>(sc.field_rows + pattern);
      e.n_main = static_cast<uint8_t>(nf + 1);
      e.n_hand = static_cast<uint8_t>(__popc(hands));
    }
  }

  constexpr int kTokensPerWarp = 32 / kSliceF4;
  const int sub = lane / kSliceF4, col = lane % kSliceF4;
  for (int slice = s_begin; slice < s_end; ++slice) {
    const int buf = (slice - s_begin) & 1;
    if (slice + 1 < s_end) {
      load_slice(slice + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // this slice (and, on the first pass, every token's ids) is in place
    const float4* tab = slices + buf * total_rows * kSliceF4 + col;
    const int c = slice * kSliceF4 + col;
    const LookupColumn dst = out.x_blk && c < width4 ? lookup_column(out, c) : LookupColumn{nullptr, 0};
    for (int t = warp * kTokensPerWarp + sub; t < count; t += (kEmbedThreads / 32) * kTokensPerWarp) {
      const EmbedIds& e = ids[t];
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < e.n_main; ++k) {
        const float4 v = tab[e.row[k] * kSliceF4];
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      if (e.n_hand) {
        float4 hand = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < e.n_hand; ++k) {
          const float4 v = tab[e.row[kEmbedMain + k] * kSliceF4];
          hand.x += v.x;
          hand.y += v.y;
          hand.z += v.z;
          hand.w += v.w;
        }
        acc.x += hand.x;
        acc.y += hand.y;
        acc.z += hand.z;
        acc.w += hand.w;
      }
      if (c < width4) {
        const int64_t token = first + t;
        if (dst.base)
          dst.base[(token >> 7) * dst.tile_stride + (token & 127)] = acc;
        else
          reinterpret_cast<float4*>(out.rows + token * width)[c] = acc;
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
}

int check_schema(const cg_plump_schema* sc) {
  CG_REQUIRE(sc, "NULL plump schema");
  CG_REQUIRE(sc->field_count > 0 && sc->field_count <= 16, "field_count must be 1..16");
  CG_REQUIRE(sc->hand_slots >= 0 && sc->hand_slots <= 16, "hand_slots must be 0..16");
  CG_REQUIRE(sc->token_width > 0 && sc->field_rows > 0 && sc->pattern_rows > 0, "bad schema sizes");
  CG_REQUIRE(sc->num_ranks > 0 && sc->num_cards > 0, "bad card counts");
  return CG_OK;
}

int embed(const cg_plump_schema& sc, const float* table, int width, const void* tokens, int token_dtype, int64_t n,
          const EmbedOut& dest, cudaStream_t s) {
  float* out = dest.rows;
  if (n == 0) return CG_OK;
  const int total_rows = sc.field_rows + sc.pattern_rows;
  // Widest slice whose two buffers fit next to the ids: 16 float4 (64 columns) for plump.
  int slice_f4 = 16;
  while (slice_f4 > 4 && embed_smem_bytes(total_rows, slice_f4, kEmbedMaxTokens, sc.token_width) > 227 * 1024)
    slice_f4 /= 2;
  const bool sliced = (width % 4) == 0 &&
                      embed_smem_bytes(total_rows, slice_f4, kEmbedMaxTokens, sc.token_width) <= 227 * 1024 &&
                      (reinterpret_cast<uintptr_t>(table) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                      sc.hand_slots * 2 <= 32 && sc.field_count <= 16;
  if (dest.x_blk && !sliced) return set_error(CG_ERR_ARGUMENT, "blocked field-lookup output needs the sliced kernel");
  if (!sliced) {
    const int64_t blocks = (n + 7) / 8;
    plump_embed_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(sc, table, width, tokens, token_dtype, n, out);
    return check_launch("plump_embed_kernel");
  }
  // Work of a CTA ~ its slices x its token passes (32 / slice_f4 tokens per warp, 16 warps):
  // pick the column-group count whose slowest CTA does the least, with one wave of CTAs.
  const int n_slices = (width / 4 + slice_f4 - 1) / slice_f4;
  const int64_t pass_tokens = static_cast<int64_t>(kEmbedThreads / 32) * (32 / slice_f4);
  int groups = 1;
  int64_t per = 0, best = -1;
  for (int gcount = 1; gcount <= 4 && gcount <= n_slices; ++gcount) {
    const int64_t token_blocks = sm_count() / gcount;
    if (token_blocks < 1) break;
    int64_t tokens = (n + token_blocks - 1) / token_blocks;
    if (tokens > kEmbedMaxTokens) tokens = kEmbedMaxTokens;
    const int64_t waves = ((n + tokens - 1) / tokens * gcount + sm_count() - 1) / sm_count();
    const int64_t work = waves * ((n_slices + gcount - 1) / gcount) * ((tokens + pass_tokens - 1) / pass_tokens);
    if (best < 0 || work < best) {
      best = work;
      groups = gcount;
      per = tokens;
    }
  }
  const int slices_per = (n_slices + groups - 1) / groups;
  const int64_t blocks = (n + per - 1) / per;
  const size_t smem = embed_smem_bytes(total_rows, slice_f4, static_cast<int>(per), sc.token_width);
  auto launch = [&](auto kernel) {
    static size_t configured[64] = {0};
    int device = 0;
    cudaGetDevice(&device);
    if (configured[device & 63] < smem) {
      cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
      if (err != cudaSuccess) return set_error(CG_ERR_CUDA, "plump_embed_sliced_kernel smem: %s", cudaGetErrorString(err));
      configured[device & 63] = smem;
    }
    return launch_pdl("plump_embed_sliced_kernel", kernel,
                      dim3(static_cast<unsigned>(blocks), static_cast<unsigned>(groups)), dim3(kEmbedThreads), smem,
                      s, sc, table, width, tokens, token_dtype, n, static_cast<int>(per), slices_per, dest);
  };
  if (slice_f4 == 16) return launch(plump_embed_sliced_kernel<16>);
  if (slice_f4 == 8) return launch(plump_embed_sliced_kernel<8>);
  return launch(plump_embed_sliced_kernel<4>);
}

struct PlumpWorkspace {
  float* lookup;
  float* ple;
  float* values;
  unsigned char* step;
  int64_t step_bytes;
  int64_t total;
};

PlumpWorkspace plan_plump(const cg_trunk_dims& dims, int64_t batch, int steps, int precision, unsigned char* base) {
  PlumpWorkspace w{};
  const int64_t nt = batch * steps;
  const int64_t d = dims.d_model, ple_w = static_cast<int64_t>(dims.n_layers) * dims.per_layer_dim;
  const int64_t val_w = static_cast<int64_t>(value_layer_count(dims)) * dims.n_kv_heads * head_dim(dims);
  int64_t at = 0;
  auto take = [&](int64_t bytes) {
    unsigned char* here = base ? base + at : nullptr;
    at = align_up(at + bytes);
    return here;
  };
  w.lookup = reinterpret_cast<float*>(take(nt * (d + ple_w + val_w) * 4));
  w.ple = reinterpret_cast<float*>(take(nt * ple_w * 4));
  w.values = reinterpret_cast<float*>(take(nt * val_w * 4));
  w.step_bytes = cg_trunk_step_workspace_bytes(&dims, batch, steps, precision);
  w.step = take(w.step_bytes);
  w.total = at;
  return w;
}

}  // namespace cg

extern "C" int cg_plump_embed(const cg_plump_schema* schema, const float* table, int width, const void* tokens,
                              int token_dtype, int64_t n_tokens, float* out, void* stream) {
  using namespace cg;
  int rc;
  if ((rc = check_schema(schema))) return rc;
  CG_REQUIRE(token_dtype == CG_I16 || token_dtype == CG_I32 || token_dtype == CG_I64, "bad token dtype");
  CG_REQUIRE(width > 0, "bad width");
  if (n_tokens == 0) return CG_OK;
  CG_REQUIRE(table && tokens && out, "cg_plump_embed: NULL pointer");
  EmbedOut dest{};
  dest.rows = out;
  return embed(*schema, table, width, tokens, token_dtype, n_tokens, dest, static_cast<cudaStream_t>(stream));
}

extern "C" int64_t cg_plump_step_workspace_bytes(const cg_trunk_dims* dims, int64_t batch, int steps, int precision) {
  if (!dims) return -1;
  return cg::plan_plump(*dims, batch, steps, precision, nullptr).total;
}

extern "C" int cg_plump_forward_ragged(const cg_trunk_dims* dims, const void* blob, const cg_plump_schema* schema,
                                       const float* table, const void* tokens, int token_dtype, int64_t batch,
                                       int steps, const int64_t* positions, const int64_t* readout_offsets,
                                       const int64_t* rows, int span, void* k_pool, void* v_pool, int kv_dtype,
                                       int64_t capacity, int max_len, int precision, void* workspace,
                                       int64_t workspace_bytes, float* hidden_out, void* stream) {
  using namespace cg;
  int rc;
  if ((rc = check_schema(schema))) return rc;
  CG_REQUIRE(dims, "NULL trunk dims");
  CG_REQUIRE(token_dtype == CG_I16 || token_dtype == CG_I32 || token_dtype == CG_I64, "bad token dtype");
  if (batch == 0) return CG_OK;
  CG_REQUIRE(table && tokens && workspace, "cg_plump_forward_ragged: NULL pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  PlumpWorkspace w = plan_plump(*dims, batch, steps, precision, static_cast<unsigned char*>(workspace));
  if (workspace_bytes < w.total)
    return set_error(CG_ERR_WORKSPACE, "plump step workspace %lld < %lld bytes", (long long)workspace_bytes,
                     (long long)w.total);
  const int64_t nt = batch * steps;
  const int ple_w = dims->n_layers * dims->per_layer_dim;
  const int val_w = value_layer_count(*dims) * dims->n_kv_heads * head_dim(*dims);
  const int width = dims->d_model + ple_w + val_w;
  const int total_rows = schema->field_rows + schema->pattern_rows;
  if (precision == CG_PREC_BF16 && tc_layers_available(*dims) && 2LL * total_rows * 4 * 16 <= 200 * 1024 &&
      schema->hand_slots * 2 <= 32 && (reinterpret_cast<uintptr_t>(table) & 15) == 0) {
    // Tensor-core path: the lookup writes its raw streams straight into the first dense
    // kernel's blocked inputs (x, per-layer PLE, value streams), which conditions them.
    EmbedOut dest{};
    dest.d = dims->d_model;
    dest.ple_w = ple_w;
    dest.P = dims->per_layer_dim;
    dest.kvw = dims->n_kv_heads * head_dim(*dims);
    tc_input_streams(*dims, batch, steps, step_tc_scratch(*dims, batch, steps, precision, w.step), &dest.x_blk,
                     &dest.ple_blk, &dest.val_blk, &dest.ntiles);
    if ((rc = embed(*schema, table, width, tokens, token_dtype, nt, dest, s))) return rc;
    return forward_ragged_impl(dims, blob, nullptr, nullptr, nullptr, batch, steps, positions, readout_offsets, rows,
                               span, k_pool, v_pool, kv_dtype, capacity, max_len, precision, w.step, w.step_bytes,
                               hidden_out, s, false, true);
  }
  EmbedOut rows_out{};
  rows_out.rows = w.lookup;
  if ((rc = embed(*schema, table, width, tokens, token_dtype, nt, rows_out, s))) return rc;
  // The residual stream x is the first buffer of the step workspace.
  float* x = reinterpret_cast<float*>(w.step);
  if ((rc = cg_trunk_condition(dims, blob, w.lookup, nt, x, w.ple, w.values, precision, s))) return rc;
  return forward_ragged_impl(dims, blob, x, w.ple, w.values, batch, steps, positions, readout_offsets, rows, span,
                             k_pool, v_pool, kv_dtype, capacity, max_len, precision, w.step, w.step_bytes, hidden_out, s,
                             true, false);
}
